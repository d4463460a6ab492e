"""The GPU norm + quantisation steps (w8a8_rmsnorm_pack_dyntok, w8a8_post_op_ffn_pack) against
the C restatement pinned to the reference: bit-identical int8 rows, ratios, normalised rows and
residual rows, for several token counts and row widths (including tails and the widest row)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from romanaccio_b200.norm import post_op_ffn_pack, rmsnorm_pack_dyntok

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,C", [(1, 1536), (1, 576), (3, 1537), (8, 2048), (2, 8960),
                                 (1, 12288), (5, 3)])
def test_rmsnorm_pack_matches_oracle(ctx, T, C):
    rng = np.random.default_rng(T * 100 + C)
    h = (rng.standard_normal((T, C)) * rng.uniform(0.1, 30)).astype(np.float32)
    h[0, : min(C, 4)] *= 50  # an outlier channel
    norm = (rng.standard_normal(C) * 0.4 + 1).astype(np.float32)
    smooth = (rng.random(C) * 3 + 0.02).astype(np.float32)
    q, ratio, u = rmsnorm_pack_dyntok(ctx, torch.from_numpy(h).cuda(),
                                      torch.from_numpy(smooth).cuda(), 6.0,
                                      norm=torch.from_numpy(norm).cuda())
    wq, wr, wu = O.rmsnorm_pack_dyntok(h, norm, smooth, 6.0)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(ratio.cpu().numpy(), wr)
    assert np.array_equal(u.cpu().numpy(), wu)
    # without the normalised-row output
    q2, r2, u2 = rmsnorm_pack_dyntok(ctx, torch.from_numpy(h).cuda(),
                                     torch.from_numpy(smooth).cuda(), 6.0)
    assert u2 is None and np.array_equal(q2.cpu().numpy(), wq)
    ctx.check()


@pytest.mark.parametrize("T,C", [(1, 1536), (4, 2049), (2, 8960)])
def test_post_op_ffn_pack_matches_oracle(ctx, T, C):
    rng = np.random.default_rng(C + T)
    op = (rng.standard_normal((T, C)) * 6).astype(np.float32)
    post = (rng.standard_normal(C) * 0.3 + 1).astype(np.float32)
    h = (rng.standard_normal((T, C)) * 3).astype(np.float32)
    ffn = (rng.random(C) * 30).astype(np.float32)
    m, q = post_op_ffn_pack(ctx, *(torch.from_numpy(a).cuda() for a in (op, post, h, ffn)))
    wm, wq = O.post_op_ffn_pack(op, post, h, ffn)
    assert np.array_equal(m.cpu().numpy(), wm)
    assert np.array_equal(q.cpu().numpy(), wq)
    ctx.check()
