"""Times the REFERENCE's own CUDA kernels (deploy/joyomni_ops compiled into
oracle/_ref by oracle/build_ref.py) on the BASELINE shapes, on this GPU.
Test/measurement infrastructure only: bench.py runs it in a subprocess because
the reference library registers the same torch.ops namespace as our shim.

    python oracle/time_ref_gpu.py oracle/_ref/joyomni_ref.so   -> one JSON line
"""
import json
import sys

import torch


def gtime(fns, reps=5):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2] / len(fns)


def main(lib):
    torch.ops.load_library(lib)
    ops = torch.ops.joyomni_ops
    dev = torch.device("cuda:0")
    gen = torch.Generator(device="cpu").manual_seed(1)
    out = {"what": "reference joyomni_ops kernels (oracle/_ref), same box, CUDA-graph timed"}
    L, H, D = 2048, 40, 128
    R = 3
    qs = [torch.randn(1, L * H, D, generator=gen).to(torch.bfloat16).to(dev) for _ in range(R)]
    ks = [torch.randn(1, L * H, D, generator=gen).to(torch.bfloat16).to(dev) for _ in range(R)]
    w = torch.ones(D, dtype=torch.bfloat16, device=dev)
    cs = torch.rand(L, D // 2, generator=gen).to(torch.bfloat16).to(dev)
    ms = gtime([(lambda j: (lambda: ops.fused_qk_norm_rope_3d_paired(qs[j], ks[j], L, H, 1e-6, w, w, cs, cs)))(i % R)
                for i in range(20)])
    out["cfg1_qk_norm_rope"] = {"us": round(ms * 1e3, 2), "GB/s": round((4 * L * H * D * 2) / (ms * 1e-3) / 1e9, 1)}
    del qs, ks
    M, N = 10530, 5120
    x = torch.randn(M, N, generator=gen).to(torch.bfloat16).to(dev)
    sc = (0.1 * torch.randn(M, N, generator=gen)).to(torch.bfloat16).to(dev)
    sh = (0.1 * torch.randn(M, N, generator=gen)).to(torch.bfloat16).to(dev)
    ms = gtime([lambda: ops.fused_norm_scale_shift(x, None, None, sc, sh, 0, 1e-6) for _ in range(10)])
    out["cfg2_norm_scale_shift_layer_MxN"] = {"us": round(ms * 1e3, 2),
                                              "GB/s": round(4 * M * N * 2 / (ms * 1e-3) / 1e9, 1)}
    ms_rms = gtime([lambda: ops.fused_norm_scale_shift(x, None, None, sc, sh, 1, 1e-6) for _ in range(10)])
    out["cfg2_norm_scale_shift_rms_MxN"] = {"us": round(ms_rms * 1e3, 2)}
    kx = torch.randn(M * 40, 128, generator=gen).to(torch.bfloat16).to(dev)
    ms = gtime([lambda: ops.rmsnorm(kx, w, 1e-6) for _ in range(10)])
    out["k3_rmsnorm_421200x128"] = {"us": round(ms * 1e3, 2),
                                   "GB/s": round(2 * kx.numel() * 2 / (ms * 1e-3) / 1e9, 1)}
    del kx
    if hasattr(ops, "sgl_per_token_quant_fp8"):
        q = torch.empty((M, N), dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty((M, 1), dtype=torch.float32, device=dev)
        ms_q = gtime([lambda: ops.sgl_per_token_quant_fp8(x, q, s) for _ in range(10)])
        out["cfg2_per_token_quant"] = {"us": round(ms_q * 1e3, 2),
                                       "GB/s": round((3 * M * N + 4 * M) / (ms_q * 1e-3) / 1e9, 1)}
        # config 2 as the reference model runs it: expand+contiguous of the [N] modulation,
        # fused_norm_scale_shift, then per-token quant (sgl_fused_ops.py:44-54, fp8_linear.py:143-167)
        w5 = torch.ones(N, dtype=torch.bfloat16, device=dev)
        sv = (0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16).to(dev)

        def chain():
            sce = sv.expand(M, N).contiguous()
            she = sv.expand(M, N).contiguous()
            y = ops.fused_norm_scale_shift(x, w5, None, sce, she, 1, 1e-6)
            ops.sgl_per_token_quant_fp8(y, q, s)
        ms_c = gtime([chain for _ in range(5)])
        out["cfg2_reference_chain_expand_norm_quant"] = {
            "us": round(ms_c * 1e3, 2),
            "GB/s_algorithmic": round((3 * M * N + 4 * M + 6 * N) / (ms_c * 1e-3) / 1e9, 1)}
    if hasattr(ops, "fp8_scaled_mm"):
        K = N
        aq = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=dev)
        sa = torch.empty((M, 1), dtype=torch.float32, device=dev)
        ops.sgl_per_token_quant_fp8(x, aq, sa)
        for name, NN, gelu in (("cfg3a_fp8_gemm_qkv_bias", 15360, False),
                               ("cfg3b_fp8_gemm_ffn_up_bias", 13824, False),
                               ("cfg3b_fp8_gemm_ffn_up_bias_then_gelu", 13824, True)):
            wq = (torch.randn(NN, K, generator=gen) * 30).clamp(-448, 448).to(torch.float8_e4m3fn).to(dev).t()
            sb = (torch.rand(NN, generator=gen) * 1e-3).to(dev)
            bias = (0.01 * torch.randn(NN, generator=gen)).to(torch.bfloat16).to(dev)
            if gelu:
                f = lambda: torch.nn.functional.gelu(ops.fp8_scaled_mm(aq, wq, sa, sb, torch.bfloat16, bias),  # noqa
                                                     approximate="tanh")
            else:
                f = lambda: ops.fp8_scaled_mm(aq, wq, sa, sb, torch.bfloat16, bias)  # noqa: E731
            ms = gtime([f for _ in range(5)])
            fl = 2.0 * M * NN * K
            out[name] = {"us": round(ms * 1e3, 2), "tflops": round(fl / (ms * 1e-3) / 1e12, 1)}
    print(json.dumps(out))


if __name__ == "__main__":
    main(sys.argv[1])
