"""Times one kernel of the forward in isolation at a workload's shapes, through
the library's kernel-level C ABI (gpt2k_*), for per-kernel roofline numbers
and small, single-kernel ncu captures.

  python mlir-learning_b200/kernel_bench.py attention --batch 64 --seq 1024 [--causal 0 --lengths uniform]
  python mlir-learning_b200/kernel_bench.py gemm --m 65536 --n 3072 --k 768 --epi 2
  python mlir-learning_b200/kernel_bench.py gemm --dtype 0 --m 8192 --n 768 --k 3072 --epi 3
  python mlir-learning_b200/kernel_bench.py layernorm --rows 65536 --d 768
  python mlir-learning_b200/kernel_bench.py decode --batch 1 --seq 128 --new 64 --dtype 1
  python mlir-learning_b200/kernel_bench.py forward --batch 1 --seq 5 --dtype 0

Inputs are seeded random device tensors; each run does --warmup untimed and
--iters timed launches between CUDA events on one stream and prints one JSON
line with the average launch time and the achieved rate against the
algorithmic work (attention: 4*H*64*S*S/2-ish causal or S*len non-causal
FLOP; GEMM: 2*M*N*K FLOP; LayerNorm: T*d*(2+2) + 2*d*4 bytes).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _pkg():
    name = "mlir_learning_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _time(torch, fn, warmup, iters):
    st = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(iters):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["attention", "gemm", "layernorm", "decode", "forward"])
    ap.add_argument("--new", type=int, default=64, help="decode: tokens generated per sequence")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--causal", type=int, default=1)
    ap.add_argument("--lengths", choices=["full", "uniform"], default="full",
                    help="uniform: right-padded, valid lengths uniform in [64, seq] (seeded)")
    ap.add_argument("--dtype", type=int, default=1,
                    help="0 f32 (attention, gemm), 1 bf16 tcgen05")
    ap.add_argument("--m", type=int, default=65536)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--epi", type=int, default=1)
    ap.add_argument("--bn", type=int, default=256)
    ap.add_argument("--out-f32", type=int, default=0)
    ap.add_argument("--b-nk", type=int, default=0, help="gemm --dtype 0: B given as [N, K]")
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--d", type=int, default=768)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()

    import numpy as np
    import torch
    pkg = _pkg()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(1234)
    st = torch.cuda.current_stream().cuda_stream
    out = {"kernel": args.kernel}
    if args.kernel == "attention":
        B, S, H = args.batch, args.seq, args.heads
        dt = torch.bfloat16 if args.dtype else torch.float32
        qkv = torch.randn(B * S, 3 * H * 64, device="cuda", generator=g).to(dt)
        o = torch.empty(B * S, H * 64, device="cuda", dtype=dt)
        mask = None
        lens = np.full(B, S)
        if args.lengths == "uniform":
            rng = np.random.default_rng(1234)
            lens = rng.integers(min(64, S), S + 1, size=B)
            mask = torch.from_numpy((np.arange(S)[None, :] < lens[:, None]).astype(np.int64)).cuda()
        ws = torch.empty(pkg.k_attention_ex_workspace_bytes(B, S), dtype=torch.uint8, device="cuda")
        mp = mask.data_ptr() if mask is not None else None
        fn = lambda: pkg.k_attention_ex(qkv.data_ptr(), mp, o.data_ptr(), B, S, H, args.dtype, args.causal,  # noqa
                                        ws.data_ptr(), st)
        ms = _time(torch, fn, args.warmup, args.iters)
        flop = 4.0 * B * H * 64 * S * (S + 1) / 2 if args.causal else 4.0 * H * 64 * S * float(lens.sum())
        out.update(B=B, S=S, H=H, causal=args.causal, lengths=args.lengths, dtype=args.dtype, ms=ms,
                   tflops=flop / ms / 1e9, algorithmic_flop=flop)
    elif args.kernel == "gemm" and args.dtype == 0:
        # The exact-FP32 SIMT GEMM: B [K, N] as the FP32 forward's Conv1D weights (--b-nk 1: [N, K], the lm_head).
        M, N, K = args.m, args.n, args.k
        A = torch.randn(M, K, device="cuda", generator=g)
        Bw = torch.randn(*((N, K) if args.b_nk else (K, N)), device="cuda", generator=g) * 0.05
        bias = torch.randn(N, device="cuda", generator=g)
        ldc = (N + 3) // 4 * 4
        C = torch.zeros(M, ldc, device="cuda")
        fn = lambda: pkg.k_gemm_f32(A.data_ptr(), Bw.data_ptr(), args.b_nk, C.data_ptr(), M, N, K, ldc,  # noqa
                                    bias.data_ptr(), C.data_ptr(), args.epi, st)
        ms = _time(torch, fn, args.warmup, args.iters)
        out.update(M=M, N=N, K=K, epi=args.epi, b_nk=args.b_nk, dtype=0, ms=ms, tflops=2.0 * M * N * K / ms / 1e9)
    elif args.kernel == "gemm":
        M, N, K = args.m, args.n, args.k
        A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        Bw = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
        bias = torch.randn(N, device="cuda", generator=g)
        ldc = (N + 7) // 8 * 8
        C = torch.zeros(M, ldc, device="cuda", dtype=torch.float32 if args.out_f32 else torch.bfloat16)
        if args.epi in (pkg.EPI_LN_BIAS, pkg.EPI_LN_BIAS_GELU, pkg.EPI_BIAS_RESID_STATS):
            # the folded-LayerNorm epilogues: c1 / c2 vectors and A's row statistics, or C's
            nv = (N + 255) // 256 * 256
            c1 = torch.randn(nv, device="cuda", generator=g)
            c2 = torch.randn(nv, device="cuda", generator=g)
            nseg = (max(K, N) + pkg.LN_SEG - 1) // pkg.LN_SEG
            stats = torch.rand(M, nseg, 2, device="cuda", generator=g) + 1.0
            fn = lambda: pkg.k_gemm_bf16_ln(A.data_ptr(), Bw.data_ptr(), C.data_ptr(), M, N, K, ldc,  # noqa
                                            args.out_f32, bias.data_ptr(), C.data_ptr(), args.epi, args.bn,
                                            c1.data_ptr(), c2.data_ptr(), stats.data_ptr(), stats.data_ptr(),
                                            1e-5, st)
        else:
            fn = lambda: pkg.k_gemm_bf16(A.data_ptr(), Bw.data_ptr(), C.data_ptr(), M, N, K, ldc,  # noqa
                                         args.out_f32, bias.data_ptr(), C.data_ptr(), args.epi, args.bn, st)
        ms = _time(torch, fn, args.warmup, args.iters)
        out.update(M=M, N=N, K=K, epi=args.epi, bn=args.bn, out_f32=args.out_f32, ms=ms,
                   tflops=2.0 * M * N * K / ms / 1e9)
    elif args.kernel == "forward":
        # The whole forward through the device entry point (repeat calls replay one CUDA graph), GPT-2 small
        # with seeded weights; --dtype 0 FP32, 1 BF16.  Logits rows padded to a 16-byte multiple.
        B, S = args.batch, args.seq
        pkg.init(pkg.gpt2_small(args.dtype), 0)
        pkg.init_seeded(1234, 0)
        ids = torch.from_numpy(pkg.seeded_ids(B, S, 1234, 50257)).cuda()
        ld = 50260
        logits = torch.empty(B * S, ld, device="cuda")
        fn = lambda: pkg.forward_device(ids.data_ptr(), None, B, S, logits.data_ptr(), ld, st)  # noqa
        ms = _time(torch, fn, args.warmup, args.iters)
        out.update(B=B, S=S, dtype=args.dtype, ms=ms, tokens_per_s=B * S / ms * 1e3)
    elif args.kernel == "decode":
        # Greedy generation with the KV cache on GPT-2 small (seeded weights): the time per
        # generated token is the difference between n_new and 1 new tokens, per step of B tokens.
        import time
        B, S, n = args.batch, args.seq, args.new
        pkg.init(pkg.gpt2_small(args.dtype), 0)
        pkg.init_seeded(1234, 0)
        prompt = pkg.seeded_ids(B, S, 1234, 50257)

        def run(k):
            t0 = time.perf_counter()
            pkg.generate(prompt, k)
            return time.perf_counter() - t0
        for _ in range(args.warmup):
            run(n)
        t1 = min(run(1) for _ in range(3))
        tn = min(run(n) for _ in range(3))
        step = (tn - t1) / (n - 1)
        out.update(B=B, S=S, new=n, dtype=args.dtype, prefill_plus_first_ms=1e3 * t1, ms_per_step=1e3 * step,
                   tokens_per_s=B / step)
    else:
        T, d = args.rows, args.d
        x = torch.randn(T, d, device="cuda", generator=g).bfloat16()
        y = torch.empty_like(x)
        gain = torch.ones(d, device="cuda")
        shift = torch.zeros(d, device="cuda")
        fn = lambda: pkg.k_layernorm(x.data_ptr(), gain.data_ptr(), shift.data_ptr(), y.data_ptr(), T, d,  # noqa
                                     1e-5, 1, st)
        ms = _time(torch, fn, args.warmup, args.iters)
        out.update(T=T, d=d, ms=ms, gbs=(T * d * 4 + 2 * d * 4) / ms / 1e6)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
