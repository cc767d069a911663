"""The quantized linears of one MTP draft step and the verify step captured
as one CUDA graph (src/mtp.zig:137-191 mtpForward, :181-191 mtpDraftLogits;
src/engine.zig:548 and :656 the M = 2 / 3 verify through lm_head), at the
model's shapes, nvfp4.

Capture needs every entry point on the path to be allocation- and
sync-free; a replay must give the eager results bit for bit (the
kernels are deterministic, including the stream-K reductions and the
argmax / logsumexp merges).  The step's outputs are also checked against
the CPU oracle, each linear on the input it actually read: fc (K = 10240),
q / k / v, o_proj, the SwiGLU pair, down, and the M = 1 draft / M = 3
verify sampling through the whole 248320-row lm_head.  The weights are
random packed bytes made on the GPU (every E2M1 code, finite scales).
"""
import numpy as np
import pytest

import qmm

pytestmark = pytest.mark.gpu

H, FFN, VOCAB = 5120, 17408, 248320


def rand_weight(n, k, dev, seed):
    """nvfp4 [n, k]: random codes, UE4M3 scales in [2^-7, 2^-3) (finite)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    codes = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, device=dev, dtype=torch.int64).to(torch.int32)
    scales = torch.randint(0x18, 0x38, (n, k // 16), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    return codes, scales


def build_step(dev, raw=None):
    """Weights of the MTP head linears and lm_head (shapes from the model:
    fc 10240 -> 5120, q_proj 5120 -> 12288, k/v 5120 -> 1024, o_proj
    6144 -> 5120, gate/up 5120 -> 17408, down 17408 -> 5120, lm_head
    5120 -> 248320).  `raw`, when given, receives each weight's packed
    (codes, scales) device tensors ("gate" / "up" for the SwiGLU pair)."""
    shapes = {"fc": (H, 2 * H), "q": (12288, H), "k": (1024, H), "v": (1024, H), "o": (H, 6144),
              "down": (H, FFN), "lm_head": (VOCAB, H)}
    w = {}
    for i, (name, (n, k)) in enumerate(shapes.items()):
        cs = rand_weight(n, k, dev, i)
        w[name] = qmm.QuantizedWeight(*cs, "nvfp4")
        if raw is not None:
            raw[name] = cs
    gate, up = rand_weight(FFN, H, dev, 20), rand_weight(FFN, H, dev, 21)
    w["mlp"] = qmm.SwiGLUWeight(*gate, *up, "nvfp4")
    if raw is not None:
        raw["gate"], raw["up"] = gate, up
    return w


def run_step(w, bufs, stream):
    """One draft step (M = 1) and the M = 3 verify logits, eager or captured.
    Non-linear ops of the model (norms, attention) are not part of this path:
    each projection reads a fixed input buffer."""
    b = bufs
    w["fc"].run(b["cat"], out=b["fused"], stream=stream)
    w["q"].run(b["fused"], out=b["q"], stream=stream)
    w["k"].run(b["fused"], out=b["k"], stream=stream)
    w["v"].run(b["fused"], out=b["v"], stream=stream)
    w["o"].run(b["attn"], out=b["o"], stream=stream)
    w["mlp"].run(b["o"], out=b["ff"], stream=stream)
    w["down"].run(b["ff"], out=b["mp"], stream=stream)
    qmm.check(qmm.lib().qmm_lm_head_argmax(w["lm_head"].handle, b["mp"].data_ptr(), 1, H, b["draft_id"].data_ptr(),
                                           b["draft_lp"].data_ptr(), None, 0, stream.cuda_stream))
    qmm.check(qmm.lib().qmm_lm_head_argmax(w["lm_head"].handle, b["verify_x"].data_ptr(), 3, H,
                                           b["verify_ids"].data_ptr(), b["verify_lp"].data_ptr(), None, 0,
                                           stream.cuda_stream))


def make_bufs(dev):
    import torch
    g = torch.Generator(device=dev).manual_seed(7)
    bf = torch.bfloat16
    return {
        "cat": torch.randn((1, 2 * H), generator=g, device=dev).to(bf),
        "fused": torch.empty((1, H), device=dev, dtype=bf),
        "q": torch.empty((1, 12288), device=dev, dtype=bf),
        "k": torch.empty((1, 1024), device=dev, dtype=bf),
        "v": torch.empty((1, 1024), device=dev, dtype=bf),
        "attn": torch.randn((1, 6144), generator=g, device=dev).to(bf),
        "o": torch.empty((1, H), device=dev, dtype=bf),
        "ff": torch.empty((1, FFN), device=dev, dtype=bf),
        "mp": torch.empty((1, H), device=dev, dtype=bf),
        "verify_x": torch.randn((3, H), generator=g, device=dev).to(bf),
        "draft_id": torch.empty((1,), device=dev, dtype=torch.int32),
        "draft_lp": torch.empty((1,), device=dev, dtype=torch.float32),
        "verify_ids": torch.empty((3,), device=dev, dtype=torch.int32),
        "verify_lp": torch.empty((3,), device=dev, dtype=torch.float32),
    }


OUTS = ("fused", "q", "k", "v", "o", "ff", "mp", "draft_id", "draft_lp", "verify_ids", "verify_lp")


def test_mtp_step_graph_replays_eager_results(cuda_device):
    import torch
    w = build_step(cuda_device)
    bufs = make_bufs(cuda_device)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        run_step(w, bufs, s)
    s.synchronize()
    eager = {k: bufs[k].clone() for k in OUTS}
    for k in OUTS:
        bufs[k].zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        run_step(w, bufs, s)
    for _ in range(3):
        for k in OUTS:
            bufs[k].zero_()
        graph.replay()
        torch.cuda.synchronize()
        for k in OUTS:
            assert torch.equal(bufs[k].view(torch.uint8) if bufs[k].dtype != torch.int32 else bufs[k],
                               eager[k].view(torch.uint8) if eager[k].dtype != torch.int32 else eager[k]), k
    qmm.device_status()
    ids = bufs["verify_ids"].cpu().numpy()
    assert np.all((ids >= 0) & (ids < VOCAB))
    del graph


def _host(cs):
    import torch
    c, sc = cs
    return c.cpu().numpy().view(np.uint32), sc.cpu().numpy()


def _bits(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_mtp_step_outputs_match_oracle(cuda_device):
    """One eager MTP step (src/mtp.zig:137-191: fc over [embed | hidden], the
    head's attention projections, MLP; src/engine.zig:548 / :656 verify
    sampling), each output against the fp64 oracle on the input the kernel
    read, and the sampled ids / log-probabilities against the oracle's greedy
    sampling of the lm_head's logits."""
    import torch
    import oracle
    from test_gpu_argmax import check_logits_and_ids
    raw = {}
    w = build_step(cuda_device, raw)
    bufs = make_bufs(cuda_device)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        run_step(w, bufs, s)
    s.synchronize()
    qmm.device_status()
    # Each linear: (weight, input buffer, output buffer).
    for name, xin, yout in (("fc", "cat", "fused"), ("q", "fused", "q"), ("k", "fused", "k"), ("v", "fused", "v"),
                            ("o", "attn", "o"), ("down", "ff", "mp")):
        codes, scales = _host(raw[name])
        ref, absref = oracle.qmm_f64_abs(_bits(bufs[xin]), codes, scales, "nvfp4")
        got = oracle.bf16_bits_to_f32(_bits(bufs[yout]))
        assert oracle.parity_violations(got, ref, absref) == 0, name
        assert oracle.rel_frobenius(got, ref) <= 2e-3, name
    # SwiGLU: h = silu(x . Wg^T) * (x . Wu^T) on the o_proj output.
    xb = _bits(bufs["o"])
    g_ref, g_abs = oracle.qmm_f64_abs(xb, *_host(raw["gate"]), "nvfp4")
    u_ref, u_abs = oracle.qmm_f64_abs(xb, *_host(raw["up"]), "nvfp4")
    assert oracle.swiglu_violations(_bits(bufs["ff"]), g_ref, u_ref, g_abs, u_abs) == 0
    # Sampling: the step's ids / log-probabilities are the greedy sample of
    # the lm_head's own logits, which meet the qmm bar.
    lm = w["lm_head"]
    codes, scales = _host(raw["lm_head"])
    for xin, id_key, lp_key in (("mp", "draft_id", "draft_lp"), ("verify_x", "verify_ids", "verify_lp")):
        ids, lp, logits = lm.argmax(bufs[xin], logits=True)
        torch.cuda.synchronize()
        step_ids, step_lp = bufs[id_key].cpu().numpy(), bufs[lp_key].cpu().numpy()
        np.testing.assert_array_equal(step_ids, ids.cpu().numpy())
        np.testing.assert_array_equal(step_lp.view(np.uint32), lp.cpu().numpy().view(np.uint32))
        check_logits_and_ids(step_ids, step_lp, logits, bufs[xin], codes, scales, "nvfp4")
    for x in w.values():
        x.close()
