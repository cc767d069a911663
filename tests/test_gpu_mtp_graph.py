"""The quantized linears of one MTP draft step and the verify step captured
as one CUDA graph (src/mtp.zig:137-191 mtpForward, :181-191 mtpDraftLogits;
src/engine.zig:548 and :656 the M = 2 / 3 verify through lm_head), at the
model's shapes, nvfp4.

Capture needs every entry point on the path to be allocation- and
sync-free; a replay must give the eager results bit for bit (the
kernels are deterministic, including the stream-K reductions and the
argmax / logsumexp merges).  The per-op numerics are covered by the
parity tests; here the weights are random packed bytes made on the GPU.
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


def build_step(dev):
    """Weights of the MTP head linears and lm_head (shapes from the model:
    fc 10240 -> 5120, q_proj 5120 -> 12288, k/v 5120 -> 1024, o_proj
    6144 -> 5120, gate/up 5120 -> 17408, down 17408 -> 5120, lm_head
    5120 -> 248320)."""
    shapes = {"fc": (H, 2 * H), "q": (12288, H), "k": (1024, H), "v": (1024, H), "o": (H, 6144),
              "down": (H, FFN), "lm_head": (VOCAB, H)}
    w = {name: qmm.QuantizedWeight(*rand_weight(n, k, dev, i), "nvfp4") for i, (name, (n, k)) in enumerate(shapes.items())}
    w["mlp"] = qmm.SwiGLUWeight(*rand_weight(FFN, H, dev, 20), *rand_weight(FFN, H, dev, 21), "nvfp4")
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
