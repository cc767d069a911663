"""lm_head with greedy sampling (src/model.zig:1300-1310 logitsOf, then
src/sample.zig:162-170 sampleToken at temp == 0) on the B200, through the C
ABI.

Bar: the logits meet the qmm parity bar against the fp64 oracle; the id is
exactly the argmax of the kernel's own bf16 logits (lowest index among
equal values) and is within the parity band of the oracle's maximum; the
log-probability matches the oracle's sequence applied to the kernel's own
logits within 1 bf16 ulp of the logsumexp (its last rounding).
"""
import numpy as np
import pytest

import oracle
import qmm

pytestmark = pytest.mark.gpu


def make_weight(n, k, mode, seed=0, scale=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * scale).astype(np.float32)
    return oracle.quantize(w, mode)


def make_x(m, k, seed=1):
    import torch
    g = torch.Generator().manual_seed(seed)
    return torch.randn((m, k), generator=g, dtype=torch.float32).to(torch.bfloat16)


def bits(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def check_sampling(w, x, codes, scales, mode):
    import torch
    ids, lp, y = w.argmax(x, logits=True)
    ids2, lp2, _ = w.argmax(x, logits=False)             # no logits written; state reset between calls
    torch.cuda.synchronize()
    qmm.device_status()
    ids, lp, ids2, lp2 = ids.cpu().numpy(), lp.cpu().numpy(), ids2.cpu().numpy(), lp2.cpu().numpy()
    np.testing.assert_array_equal(ids, ids2)
    np.testing.assert_array_equal(lp.view(np.uint32), lp2.view(np.uint32))
    check_logits_and_ids(ids, lp, y, x, codes, scales, mode)
    return ids, lp


def check_logits_and_ids(ids, lp, y, x, codes, scales, mode):
    """The logits y meet the qmm bar against the fp64 oracle; ids / lp are the
    greedy sample of those logits (lowest index among equal values; lp within
    1 bf16 ulp of the logsumexp) and each id's exact logit is within the bar
    of the exact maximum."""
    yb = bits(y)
    xb = bits(x)
    ref, absref = oracle.qmm_f64_abs(xb, codes, scales, mode)
    assert oracle.parity_violations(oracle.bf16_bits_to_f32(yb), ref, absref) == 0
    want_ids, want_lp = oracle.greedy_sample(yb)
    np.testing.assert_array_equal(ids, want_ids)
    lse_ulp = oracle.bf16_ulp(np.abs(want_lp) + 1.0)
    assert np.all(np.abs(lp - want_lp) <= lse_ulp + 1e-6), (lp, want_lp)
    # Against the fp64 reference: the chosen logit is within the bar of the max.
    for r in range(len(ids)):
        top = np.max(ref[r])
        tol = oracle.bf16_ulp(top) + 2.0 ** -20 * absref[r, ids[r]]
        assert ref[r, ids[r]] >= top - 2 * tol


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
def test_argmax_small(cuda_device, mode, m):
    n, k = 1000, 512                          # n not a multiple of the 128-row block
    codes, scales = make_weight(n, k, mode, seed=m)
    w = qmm.QuantizedWeight(codes, scales, mode)
    x = make_x(m, k, seed=m).to(cuda_device)
    check_sampling(w, x, codes, scales, mode)


@pytest.mark.parametrize("m", [1, 3])
def test_argmax_vocab_slice(cuda_device, m):
    """A 32768-row slice of the [248320, 5120] nvfp4 lm_head: many row blocks
    split across CTAs (stream-K) feed one key and one logsumexp per row."""
    n, k, mode = 32768, 5120, "nvfp4"
    codes, scales = make_weight(n, k, mode, seed=11)
    w = qmm.QuantizedWeight(codes, scales, mode)
    x = make_x(m, k, seed=m).to(cuda_device)
    check_sampling(w, x, codes, scales, mode)


def random_packed(n, k, seed):
    """nvfp4 [n, k] as random packed words (every E2M1 code) and UE4M3 scales
    in [2^-7, 2^-3): built directly, without an [n, k] fp32 draw."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 2 ** 32, (n, k // 8), dtype=np.uint32)
    scales = rng.integers(0x18, 0x38, (n, k // 16), dtype=np.uint8)
    return codes, scales


@pytest.mark.parametrize("m", [1, 3])
def test_argmax_full_vocab(cuda_device, m):
    """The whole [248320, 5120] nvfp4 lm_head (src/model.zig:1300-1310
    logitsOf, all 248320 rows) with greedy sampling, M = 1 (decode) and M = 3
    (MTP verify): every logit against the fp64 oracle, the id and log-
    probability against the oracle's sampling of the kernel's logits."""
    n, k, mode = 248320, 5120, "nvfp4"
    codes, scales = random_packed(n, k, seed=12)
    w = qmm.QuantizedWeight(codes, scales, mode)
    x = make_x(m, k, seed=20 + m).to(cuda_device)
    check_sampling(w, x, codes, scales, mode)
    w.close()


def test_argmax_ties_take_lowest_index(cuda_device):
    """Rows 5, 37, 700 and 901 are identical and carry the largest logit (x
    is the sign pattern of row 5): the id is 5, whichever CTA finishes first."""
    import torch
    n, k, mode = 1024, 256, "mxfp8"
    codes, scales = make_weight(n, k, mode, seed=3)
    for r in (37, 700, 901):
        codes[r] = codes[5]
        scales[r] = scales[5]
    w5 = oracle.dequantize(codes[5:6], scales[5:6], mode)[0]
    x = torch.from_numpy(np.where(w5 >= 0, 1.0, -1.0).astype(np.float32)[None, :]).to(torch.bfloat16)
    w = qmm.QuantizedWeight(codes, scales, mode)
    xd = x.to(cuda_device)
    for _ in range(3):
        ids, _, yy = w.argmax(xd, logits=True)
        yv = yy.float().cpu().numpy()[0]
        assert yv[5] == yv[37] == yv[700] == yv[901] == yv.max()
        assert int(ids.cpu()[0]) == 5


def test_argmax_nan_logit_wins(cuda_device):
    n, k, mode = 300, 256, "mxfp8"
    codes, scales = make_weight(n, k, mode, seed=4)
    scales[123, 0] = 0xFF                     # UE8M0 NaN: row 123 is NaN for every x
    scales[200, 1] = 0xFF
    w = qmm.QuantizedWeight(codes, scales, mode)
    ids, lp, _ = w.argmax(make_x(2, k).to(cuda_device))
    assert ids.cpu().tolist() == [123, 123]
    assert np.isnan(lp.cpu().numpy()).all()


def test_argmax_unaligned_x_and_errors(cuda_device):
    import torch
    n, k, mode = 640, 512, "nvfp4"
    codes, scales = make_weight(n, k, mode, seed=8)
    w = qmm.QuantizedWeight(codes, scales, mode)
    xbig = make_x(3, k + 8, seed=2).to(cuda_device)
    x = xbig[:, 2:2 + k]                       # 4-byte aligned rows: the unfused path
    ids, lp, y = w.argmax(x, logits=True)
    torch.cuda.synchronize()
    want_ids, want_lp = oracle.greedy_sample(bits(y))
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids)
    assert np.all(np.abs(lp.cpu().numpy() - want_lp) <= oracle.bf16_ulp(np.abs(want_lp) + 1.0) + 1e-6)
    with pytest.raises(qmm.QmmError) as ei:
        w.argmax(make_x(9, k).to(cuda_device))
    assert ei.value.name == "BadShape"
