"""The persistent decode-chain kernel (one cooperative launch for a whole stack of linears and
the LM-head top-k) must produce exactly the per-linear path's outputs, which are themselves
bit-exact against the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth
from romanaccio_b200.chain import ChainStepSpec, DecodeChain
from romanaccio_b200.decode import DecodeStack

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,T,layers,vocab", [
    (synth.SMOLLM_135M, 1, 3, 49152),
    (synth.SMOLLM_135M, 3, 2, 8192),
    (synth.QWEN25_15B, 1, 2, 151936),
    (synth.QWEN25_15B, 8, 1, 20000),
    (synth.GEMMA_12B, 1, 1, 32768),
])
def test_chain_matches_per_linear_path(ctx, shape, T, layers, vocab):
    st = DecodeStack(ctx, shape, T, layers=layers, lm_vocab=vocab, use_chain=True, seed=3)
    x = synth.activations(T, shape.hidden, seed=5).to(st.dev)
    st.x.copy_(x)
    # every step reads the previous step's output (the LM head is the chain's last step for T = 1)
    assert st.chain.barriers == 4 * layers - (0 if st.chain_lm else 1)
    st.run_device()
    torch.cuda.synchronize()
    chain_outs = [o.clone() for o in st.outs]
    chain_val, chain_idx = st.top_val.clone(), st.top_idx.clone()
    # per-linear launches over the same buffers
    st.run_linears()
    st.run_lm_head()
    torch.cuda.synchronize()
    for a, b in zip(chain_outs, st.outs):
        assert torch.equal(a, b)
    assert torch.equal(chain_idx, st.top_idx)
    assert torch.equal(chain_val, st.top_val)
    # and against the oracle: the final hidden state's LM head
    h = st.outs[3].cpu().numpy()
    wq, acc_step = st.lm_host
    lg = O.dequant_acc(O.gemm_i32(O.emb_norm_pack(h, *st.lm_norm), wq), acc_step)
    wv, wi = O.topk(lg, st.k)
    assert np.array_equal(chain_idx.cpu().numpy(), wi)
    assert np.array_equal(chain_val.cpu().numpy(), wv)
    # repeated launches are stable (arrival counters and top-k counter reset correctly)
    for _ in range(5):
        st.run_device()
    torch.cuda.synchronize()
    assert torch.equal(st.top_idx, chain_idx)
    ctx.check()


@pytest.mark.parametrize("shape,T,vocab", [(synth.SMOLLM_135M, 3, 8192), (synth.QWEN25_15B, 8, 20000)])
def test_chain_lm_step_with_several_tokens(ctx, shape, T, vocab):
    """The LM head as the chain's last step with several tokens (the decode stack runs it after
    the chain for T > 1, but the chain supports it): same top-k as the separate head."""
    st = DecodeStack(ctx, shape, T, layers=1, lm_vocab=vocab, use_chain=True, seed=4)
    assert not st.chain_lm
    st.x.copy_(synth.activations(T, shape.hidden, seed=6).to(st.dev))
    st.run_device()
    torch.cuda.synchronize()
    want_val, want_idx = st.top_val.clone(), st.top_idx.clone()
    chain = st._build_chain(with_lm=True)
    st.top_val.zero_()
    st.top_idx.zero_()
    chain.forward()
    torch.cuda.synchronize()
    assert torch.equal(st.top_idx, want_idx)
    assert torch.equal(st.top_val, want_val)
    chain.close()
    ctx.check()


def test_chain_oracle_chain_bit_exact(ctx):
    """Two dependent linears with requant outputs checked step by step against the oracle."""
    T = 2
    p1 = synth.make_linear(576, 1536, seed=1)
    p2 = synth.make_linear(1536, 576, seed=2)

    def lin(p):
        s = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8,
                                 in_thresh=p.in_thresh, in_step=p.in_step,
                                 in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
        return rb.W8A8Linear(ctx, p.wq, s, quant_m=p.quant_m, trunc=p.trunc, acc_step=p.acc_step)

    l1, l2 = lin(p1), lin(p2)
    x = synth.activations(T, 576, seed=9)
    xd = x.cuda()
    y1 = torch.empty((T, 1536), dtype=torch.float32, device="cuda")
    y2 = torch.empty((T, 576), dtype=torch.float32, device="cuda")
    r1 = torch.empty(T, dtype=torch.float32, device="cuda")
    r2 = torch.empty(T, dtype=torch.float32, device="cuda")
    ch = DecodeChain(ctx, [ChainStepSpec(l1, xd, y1, ratio=r1), ChainStepSpec(l2, y1, y2, ratio=r2)], T)
    assert ch.barriers == 1
    ch.forward()
    torch.cuda.synchronize()
    *_, yy1 = O.linear(x.numpy(), p1.wq, p1.quant_m, p1.trunc, p1.out_step_chan, p1.in_inv_smooth,
                       in_thresh=p1.in_thresh)
    q2, rr2, _, _, yy2 = O.linear(yy1, p2.wq, p2.quant_m, p2.trunc, p2.out_step_chan,
                                  p2.in_inv_smooth, in_thresh=p2.in_thresh)
    assert np.array_equal(y1.cpu().numpy(), yy1)
    assert np.array_equal(y2.cpu().numpy(), yy2)
    assert np.array_equal(r2.cpu().numpy(), rr2)


def test_independent_steps_need_no_barrier(ctx):
    """Steps that share an input and write disjoint outputs run without a grid barrier."""
    T, K = 1, 1536
    ps = [synth.make_linear(K, n, seed=20 + i) for i, n in enumerate((1536, 256, 256))]
    lins = []
    for p in ps:
        s = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8,
                                 in_thresh=p.in_thresh, in_step=p.in_step,
                                 in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
        lins.append(rb.W8A8Linear(ctx, p.wq, s, quant_m=p.quant_m, trunc=p.trunc))
    x = synth.activations(T, K, seed=4)
    xd = x.cuda()
    out = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
    views = [out[:, :1536], out[:, 1536:1792], out[:, 1792:]]
    ch = DecodeChain(ctx, [ChainStepSpec(l, xd, v) for l, v in zip(lins, views)], T)
    assert ch.barriers == 0
    ch.forward()
    torch.cuda.synchronize()
    for p, v in zip(ps, views):
        *_, y = O.linear(x.numpy(), p.wq, p.quant_m, p.trunc, p.out_step_chan, p.in_inv_smooth,
                         in_thresh=p.in_thresh)
        assert np.array_equal(v.cpu().numpy(), y)


# ---------------------------------------------------------------------------------------
# The benchmarked configurations end to end against the oracle's whole decode step.
_STACKS = {}


def _qwen_stack(ctx):
    if "qwen" not in _STACKS:
        _STACKS["qwen"] = DecodeStack(ctx, synth.QWEN25_15B, 1, seed=0)
    return _STACKS["qwen"]


def _oracle_step(st, x):
    from oracle.oracle import DecodeOracle
    orc = DecodeOracle(st.params_host, st.lm_oracle(), st.T, st.shape, k=st.k)
    return orc.run(x)


def _check_step(st, x):
    st.x.copy_(torch.from_numpy(x).to(st.dev))
    st.run_device()
    torch.cuda.synchronize()
    h, val, idx = _oracle_step(st, x)
    assert np.isfinite(h).all(), "the oracle's final hidden state is not finite"
    assert np.array_equal(st.outs[3].cpu().numpy(), h), "final hidden state differs"
    assert np.array_equal(st.top_idx.cpu().numpy(), idx), "top-k ids differ"
    assert np.array_equal(st.top_val.cpu().numpy(), val), "top-k values differ"
    assert np.array_equal(st.ids.cpu().numpy(), idx[:, 0]), "argmax differs"
    # the LM head sees a real distribution (its normalised input does not quantise to zeros)
    assert all(len(np.unique(val[t])) > st.k // 2 for t in range(st.T)), "tied top-k logits"


@pytest.mark.parametrize("T", [1, 8, 32])
def test_qwen_28_layer_step_matches_oracle(ctx, T):
    """Config 1 as benchmarked: all 28 layers and the 151936-row LM head with its top-40, T = 1
    and 8 through the persistent chain, T = 32 through the tensor-core linears, against the
    oracle's 28-layer step on the same input."""
    base = _qwen_stack(ctx)
    st = base if T == 1 else DecodeStack(ctx, synth.QWEN25_15B, T, seed=0, share_from=base)
    assert st.layers == 28 and st.V == 151936
    if T <= 8:
        assert st.chain is not None
    else:
        assert st.chain is None
    _check_step(st, synth.activations(T, 1536, seed=40 + T).numpy())
    ctx.check()


def test_gemma_48_layer_step_matches_oracle(ctx):
    """Config 4: 48 Gemma-12B-class layers and the 262144-row LM head, T = 1."""
    st = DecodeStack(ctx, synth.GEMMA_12B, 1, seed=0)
    _check_step(st, synth.activations(1, 3840, seed=44).numpy())
    ctx.check()


def test_smollm_30_layer_step_matches_oracle(ctx):
    """Config 0: 30 SmolLM-135M-shaped layers (smoothing from max |x|, no clamp) and the
    49152-row LM head, T = 1."""
    st = DecodeStack(ctx, synth.SMOLLM_135M, 1, seed=0, stat="max", clamp=None)
    _check_step(st, synth.activations(1, 576, seed=45).numpy())
    ctx.check()
