"""The screening kernel on CTA pairs (clusters of two SMs sharing one M = 256 MMA, each
streaming half of every center tile) against the same kernel on single SMs.

Pairs engage for tiles of 8 or more K blocks (d >= 512 for fp16/bf16 operands, d >= 256
for tf32).  The MMA results are the same either way, so the fused argmin's outputs --
labels, minimum distances and the flagged-pair count -- must be identical, including
ragged row counts (a pair's second row tile past n) and center counts.
"""
import numpy as np
import pytest
import torch

import _ops
from _lib import device_check, lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("op,n,m,d", [("fp16_fp32", 3000, 517, 512), ("bf16_fp32", 1031, 700, 640),
                                      ("tf32_fp64", 513, 300, 256), ("fp16_fp32", 1, 9, 1024),
                                      ("bf16_fp32", 300, 1024, 128)])
def test_pairs_match_single_sm(op, n, m, d):
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(n + m + d)
    C = torch.randn(m, d, generator=g, device="cuda")
    P = (C[torch.randint(0, m, (n,), generator=g, device="cuda")] + 0.3 * torch.randn(n, d, generator=g,
                                                                                      device="cuda")).contiguous()
    kappa = 0.1 if op.startswith("bf16") else 0.5
    outs = []
    try:
        for pairs in (1, 0):
            L.euc_set_screen_pairs(pairs)
            lab, md, cnt = _ops.run_argmin(op, P, C, kappa)
            device_check()
            outs.append((lab.cpu(), md.cpu(), int(cnt.item())))
    finally:
        L.euc_set_screen_pairs(1)
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    assert outs[0][2] == outs[1][2]


def test_pairs_c5b_shape_vs_oracle():
    # d = 1024, k = 8192 fp16-representable values (C5b's shape, 256 of its 2^21 rows) at
    # kappa = 0.5, where no pair is flagged: the paired screen's labels equal the
    # oracle's wherever the top-two gap exceeds the screen's resolution
    rng = np.random.default_rng(4)
    n, d, k = 256, 1024, 8192
    P = rng.normal(size=(n, d)).astype(np.float16).astype(np.float32)
    C = rng.normal(size=(k, d)).astype(np.float16).astype(np.float32)
    lab, _, cnt = _ops.run_argmin("tensorcore_fp16_fp32", torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda(), 0.5)
    device_check()
    D, flag, cnt_o, _ = O.tiled("fp16_fp32", P, C, 0.5)
    assert cnt_o == 0 and int(cnt.item()) == 0
    pp = O.norms_f32(P, "sumsq").astype(np.float64)
    sure = O.top2_gap(D) > 2.0 ** -10 * (pp + float(O.norms_f32(C, "sumsq").max()))
    assert sure.mean() > 0.5
    np.testing.assert_array_equal(lab.cpu().numpy()[sure], O.argmin_first(D)[sure])
