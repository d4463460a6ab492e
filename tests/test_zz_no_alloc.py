"""The allocation-free LM-head top-k entry point (w8a8_lmhead_topk_noalloc), called through the
C ABI, must give exactly what the regular entry point (w8a8_linear_forward_topk) gives.

It exists for callers that cannot call cudaMalloc (allocator or memory-pool callbacks, plugins
whose host owns every device allocation, paths that must not take the driver's allocation
locks): its scratch lives in a module-scope device array instead of memory allocated at
create time.  Two calls in a row check that the shared scratch, which keeps the previous call's
contents, is reset correctly.  This file is collected last, so a run that stops at the first
failure has already run every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import romanaccio_b200 as rb
from oracle import oracle as O
from romanaccio_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _noalloc(lib, w_dev, ldw, K, N, acc_dev, in_step, x_dev, T, k, row_offset):
    val = torch.full((T, k), -1.0, dtype=torch.float32, device="cuda")
    idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    st = lib.w8a8_lmhead_topk_noalloc(w_dev.data_ptr(), ldw, K, N, acc_dev.data_ptr(), in_step,
                                      x_dev.data_ptr(), x_dev.stride(0), T, k, row_offset,
                                      val.data_ptr(), idx.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert st == _lib.SUCCESS, lib.w8a8_last_error().decode()
    return val, idx


@pytest.mark.parametrize("V,K,T,k", [(151936, 1536, 1, 40), (24576, 576, 3, 64), (5000, 100, 8, 7)])
def test_noalloc_matches_regular_entry_point(ctx, V, K, T, k):
    lib = _lib.load()
    rng = np.random.default_rng(V + K)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    acc_step = (rng.random(V) * 1e-4 + 1e-6).astype(np.float32)
    in_step, row_offset = 0.029, 1234
    # regular path: a linear created (and allocated) through w8a8_linear_create
    shard = rb.LmHeadShard(ctx, wq, acc_step, in_step, row_offset=row_offset)
    # caller-owned device buffers for the allocation-free path (rows padded to 16 bytes)
    k_pad = (K + 15) // 16 * 16
    w_pad = np.zeros((V, k_pad), np.int8)
    w_pad[:, :K] = wq
    w_dev = torch.from_numpy(w_pad).cuda()
    acc_dev = torch.from_numpy(acc_step).cuda()
    for call in range(2):
        x_host = synth.activations(T, K, seed=call + T).numpy()
        x = torch.from_numpy(x_host).cuda()
        want_v, want_i = shard.forward(x, k)
        got_v, got_i = _noalloc(lib, w_dev, k_pad, K, V, acc_dev, in_step, x, T, k, row_offset)
        torch.cuda.synchronize()
        assert torch.equal(got_i, want_i), f"call {call}: ids differ"
        assert torch.equal(got_v, want_v), f"call {call}: values differ"
        # and against the oracle directly: static pack, int32 GEMM, acc * acc_step, top-k
        logits = O.dequant_acc(O.gemm_i32(O.pack_static(x_host, in_step), wq), acc_step)
        ref_v, ref_i = O.topk(logits, k, id_offset=row_offset)
        assert np.array_equal(got_i.cpu().numpy(), ref_i), f"call {call}: ids differ from the oracle"
        assert np.array_equal(got_v.cpu().numpy(), ref_v), f"call {call}: values differ from the oracle"
    ctx.check()


def test_noalloc_allocates_nothing_after_its_setup_call(ctx):
    """After the first (set-up) call on the device, further calls leave the device's free
    memory unchanged: the scratch is the module-scope array, not an allocation."""
    lib = _lib.load()
    V, K, T, k = 49152, 576, 2, 40
    rng = np.random.default_rng(11)
    w_dev = torch.from_numpy(rng.integers(-127, 128, size=(V, K)).astype(np.int8)).cuda()
    acc_dev = torch.from_numpy((rng.random(V) * 1e-4 + 1e-6).astype(np.float32)).cuda()
    x = torch.from_numpy(synth.activations(T, K, seed=5).numpy()).cuda()
    val = torch.empty((T, k), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def call():
        st = lib.w8a8_lmhead_topk_noalloc(w_dev.data_ptr(), K, K, V, acc_dev.data_ptr(), 0.03,
                                          x.data_ptr(), K, T, k, 0, val.data_ptr(),
                                          idx.data_ptr(), s)
        assert st == _lib.SUCCESS, lib.w8a8_last_error().decode()

    call()  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    lib = _lib.load()
    K, N = 20000, 256
    w_dev = torch.zeros((N, K), dtype=torch.int8, device="cuda")
    acc_dev = torch.ones(N, dtype=torch.float32, device="cuda")
    x = torch.zeros((8, K), dtype=torch.float32, device="cuda")
    out_v = torch.empty((8, 8), dtype=torch.float32, device="cuda")
    out_i = torch.empty((8, 8), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # 8 tokens x 20000 bytes exceeds the 128 KiB activation scratch
    st = lib.w8a8_lmhead_topk_noalloc(w_dev.data_ptr(), K, K, N, acc_dev.data_ptr(), 0.1,
                                      x.data_ptr(), K, 8, 8, 0, out_v.data_ptr(), out_i.data_ptr(), s)
    assert st == _lib.ERR_INVALID_ARG
    assert b"scratch" in lib.w8a8_last_error()
    # more than 8 tokens
    st = lib.w8a8_lmhead_topk_noalloc(w_dev.data_ptr(), K, 64, N, acc_dev.data_ptr(), 0.1,
                                      x.data_ptr(), K, 9, 8, 0, out_v.data_ptr(), out_i.data_ptr(), s)
    assert st == _lib.ERR_INVALID_ARG
    # The third limit, T * CTAs * (k + 1) <= 163840 candidate keys, is above what any launch
    # on a 148-SM B200 needs (at most 8 tokens * 296 CTAs * 65 = 153920 keys), so no request
    # that passes the token limit can reach it here.
    props = torch.cuda.get_device_properties(0)
    assert 8 * 2 * props.multi_processor_count * 65 <= 163840
