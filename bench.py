"""GPT-2 prefill throughput on B200: tokens/s of the GPT-2 small BF16 forward,
batch 64 x seq 1024 (global batch, split over the ranks), logits resident
on each shard.

  python bench.py [--gpus N --steps K --warmup W]        # this library
  python bench.py --impl reference [...]                  # the CPU reference path
  torchrun --nproc-per-node N bench.py --gpus N ...       # one process per GPU
  python bench.py --config 3                              # BERT-base encoder, B128 x S512

--config selects another of the reference's workloads (1: GPT-2 small FP32
B8xS1024, 3: the BERT-base BF16 encoder B128xS512 with right-padded
sequences of seeded lengths in [64, 512], 4: the GPT-2-XL shape with FP8
weight-only GEMMs B32xS1024); the default is the headline workload.

One step = one forward over this rank's share of the configuration's batch
(strong scaling by default: B/N sequences per rank; --scaling weak gives every
rank the whole batch), ids resident in HBM, FP32 logits written to HBM.
value = all ranks' tokens / max-over-ranks device time of the K timed steps
(CUDA events on the launching stream).  Every step reads and writes far more
than the 126 MB L2 (the FP32 logits alone are 13.2 GB at N=1), so no separate
L2 flush is done.

Also reported: a per-kernel event breakdown with the roofline of the
dominant kernel (scaled to the timed step), the same forward with bf16
logits, at N > 1 the forward plus the NCCL gather of every shard's logits
into rank 0, the end-to-end rate through the drop-in gpt2_decoder (host ids
in, a malloc'd FP32 result out, freed each step) and through
gpt2_forward_host with pinned buffers, the SM clocks sampled during the
timed steps, and (rank 0, N=1) the CPU oracle timed on one sequence of the
same workload.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
SEED = 1234
V, DH = 50257, 64
LD_LOGITS = 50304  # row stride of the resident logits (16-byte aligned rows)

# The workloads of the reference's configurations that run through this path:
# (name, layers, d_model, heads, d_mlp, dtype code, dtype label, global batch, seq).
CONFIGS = {
    0: ("gpt2-small FP32 prefill B1xS5, the reference host program's own call (latency)", 12, 768, 12, 3072, 0,
        "f32", 1, 5),
    1: ("gpt2-small FP32 prefill B8xS1024", 12, 768, 12, 3072, 0, "f32", 8, 1024),
    2: ("gpt2-small BF16 prefill B64xS1024", 12, 768, 12, 3072, 1, "bf16", 64, 1024),
    3: ("bert-base BF16 encoder B128xS512, valid lengths uniform in [64, 512]", 12, 768, 12, 3072, 1,
        "bf16", 128, 512),
    4: ("gpt2-xl-shape FP8 weight-only prefill B32xS1024", 48, 1600, 25, 6400, 2, "fp8w-e4m3/bf16", 32,
        1024),
}
BERT_V, BERT_P, BERT_TV = 30522, 512, 2
# The reference's one published number for this path: 2.44 s for the B1 x S5 FP32 forward of its
# host program (README.md:86, RTX 4080 Laptop GPU, its best pipeline), i.e. 5 / 2.44 tokens/s.
PUBLISHED_B1S5_TOKENS_PER_S = 5 / 2.44
METRICS = {0: "GPT-2 prefill tokens/s (GPT-2 small FP32, B1 x S5)",
           2: "GPT-2 prefill tokens/s (GPT-2 small, B64 x S1024)",
           3: "BERT-base encoder tokens/s (B128 x S512 positions, padding included)"}
L, D, H, FF = 12, 768, 12, 3072  # set from the chosen configuration in main()


def _pkg():
    name = "mlir_learning_b200"
    if name in sys.modules:
        return sys.modules[name]
    path = os.path.join(ROOT, "mlir-learning_b200", "__init__.py")
    spec = importlib.util.spec_from_file_location(name, path, submodule_search_locations=[os.path.dirname(path)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _oracle():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import oracle as O
    return O


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16": p["bf16_tflops"], "bf16_sus": p["bf16_tflops_sustained"],
                "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sus": 1400.0, "src": "fallback"}


def shard_rows(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of the global batch that `rank` of `world` processes.  Sequences are
    independent, so the batch splits with no data-path collective; the global batch must divide."""
    if world < 1 or not 0 <= rank < world or global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split over {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def max_over_ranks(seconds: float, dist=None, device=None) -> float:
    """The slowest rank's time (the job's time); identity on one rank."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return seconds
    import torch
    t = torch.tensor([seconds], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def kernel_work(B, S, config=2):
    """Algorithmic work of one launch of each kernel kind at B sequences of S tokens:
    ('flop', F) for tensor-bound kernels, ('bytes', N) for the bandwidth-bound ones.  At B1 x S5
    (config 0) every GEMM streams its FP32 weight for five rows: its bound is the weight read."""
    T = B * S
    if config == 0:
        return {
            "gemm_qkv": ("bytes", 4 * D * 3 * D + 4 * T * (D + 3 * D)),
            "gemm_proj": ("bytes", 4 * D * D + 4 * T * 3 * D),
            "gemm_fc": ("bytes", 4 * D * FF + 4 * T * (D + FF)),
            "gemm_mproj": ("bytes", 4 * FF * D + 4 * T * (FF + 2 * D)),
            "lm_head": ("bytes", 4 * V * D + 4 * T * (D + V)),
            "attention": ("bytes", 4 * T * 4 * D),
            "layernorm": ("bytes", T * D * 8 + 2 * D * 4),
            "embed": ("bytes", T * 8 + 2 * T * D * 4 + T * D * 4),
        }
    return {
        "gemm_qkv": ("flop", 2.0 * T * D * 3 * D),
        "gemm_proj": ("flop", 2.0 * T * D * D),
        "gemm_fc": ("flop", 2.0 * T * D * FF),
        "gemm_mproj": ("flop", 2.0 * T * FF * D),
        "lm_head": ("flop", 2.0 * T * D * V),
        "attention": ("flop", 4.0 * B * H * DH * S * (S + 1) / 2),
        "layernorm": ("bytes", T * D * (2 + 2) + 2 * D * 4),
        "embed": ("bytes", T * 8 + 2 * T * D * 2 + T * D * 2),
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def traffic_per_launch(config: int, kernel: str, tokens: int):
    """DRAM bytes (read + write) per launch of `kernel` at `tokens` tokens per rank, scaled by
    tokens from the ncu capture recorded in profiles/traffic.json (None if not captured)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            ent = json.load(f).get(str(config), {}).get(kernel)
        return int(ent["bytes_per_launch_captured"] * tokens / ent["captured_tokens"])
    except Exception:
        return None


# FP32 SIMT (FFMA) peak of a B200: 148 SMs x 128 FP32 lanes x 2 FLOP at the 1965 MHz maximum SM
# clock, for context; the exact-FP32 configuration is rated against the FFMA throughput measured in
# the same run (gpt2k_ffma_peak).
FP32_SIMT_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def kernel_breakdown(prof: dict, work: dict, nprof: int, peaks: dict, config: int, tokens: int,
                     ffma_tflops: float | None = None, timed_step_ms: float | None = None):
    """Per-kernel ms / share / rate of `nprof` profiled steps and the roofline of the dominant
    kernel.  The exact-FP32 workload (--config 1) runs on FFMA, not the tensor cores: its
    FLOP-bound kernels are rated against the FP32 SIMT peak.

    The profiled steps bracket every launch with events and run at higher SM clocks than the
    timed steps (which the 1000 W cap slows), so when timed_step_ms is given each kernel's
    duration is also scaled to the timed step by its share of the profiled step
    (`avg_launch_ms_at_timed_step`), and the roofline's `achieved` uses that scaled duration:
    algorithmic work per launch / (share x timed step / launches per step)."""
    kernels = {}
    for k, (ms, n) in prof.items():
        if n == 0:
            continue
        ent = {"ms_per_step": ms / nprof, "launches_per_step": n // nprof, "avg_launch_ms": ms / n}
        if k in work:
            kind, amount = work[k]
            per_launch_s = ms / n / 1000.0
            if kind == "flop":
                ent["tflops"] = amount / per_launch_s / 1e12
            else:
                ent["gbs"] = amount / per_launch_s / 1e9
        kernels[k] = ent
    step_ms = sum(e["ms_per_step"] for e in kernels.values())
    for k, e in kernels.items():
        e["share"] = e["ms_per_step"] / step_ms if step_ms else None
        if timed_step_ms and step_ms:
            e["avg_launch_ms_at_timed_step"] = e["share"] * timed_step_ms / max(1, e["launches_per_step"])
            if k in work:
                kind, amount = work[k]
                rate = amount / (e["avg_launch_ms_at_timed_step"] / 1000.0)
                e["tflops_at_timed_step" if kind == "flop" else "gbs_at_timed_step"] = rate / (1e12 if kind == "flop" else 1e9)
    dom = max(kernels, key=lambda k: kernels[k]["ms_per_step"])
    traffic = traffic_per_launch(config, dom, tokens)
    kind, amount = work.get(dom, ("flop", 0.0))
    per_launch_s = kernels[dom].get("avg_launch_ms_at_timed_step", kernels[dom]["avg_launch_ms"]) / 1000.0
    if kind == "flop" and config == 1:
        achieved = amount / per_launch_s / 1e12
        peak = ffma_tflops or FP32_SIMT_NOMINAL_TFLOPS
        roof = {"bound": "fp32-simt", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic, "kernel": dom,
                "peak_kind": ("FFMA measured in this run (gpt2k_ffma_peak, burst)" if ffma_tflops else
                              "FFMA nominal (148 SMs x 128 lanes x 2 x 1965 MHz)"),
                "ffma_nominal": FP32_SIMT_NOMINAL_TFLOPS, "algorithmic_per_launch": amount}
    elif kind == "flop":
        achieved = amount / per_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_sus"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_sus"], "traffic": traffic, "kernel": dom,
                "peak_kind": f"bf16 sustained ({peaks['src']})", "algorithmic_per_launch": amount,
                "time_basis": "profiled share x timed step" if timed_step_ms else "profiled launch events"}
    else:
        achieved = amount / per_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic, "kernel": dom,
                "peak_kind": f"hbm copy ({peaks['src']})", "algorithmic_per_launch": amount}
    return kernels, roof


def bert_lengths(global_batch: int, S: int) -> np.ndarray:
    """Seeded valid lengths of the BERT workload, uniform in [64, S] (Philox stream 0x30002)."""
    O = _oracle()
    lo = min(64, S)
    return lo + O.token_ids(1, global_batch, SEED, S - lo + 1, stream=O.BERT_IDS_STREAM + 2)[0]


def bert_kernel_work(B, S, lens):
    """Algorithmic work per launch of each BERT kernel kind for B sequences of S positions with
    valid lengths `lens`: attention counts every query row against the valid keys only."""
    T = B * S
    return {
        "gemm_qkv": ("flop", 2.0 * T * D * 3 * D),
        "gemm_attn_out": ("flop", 2.0 * T * D * D),
        "gemm_intermediate": ("flop", 2.0 * T * D * FF),
        "gemm_output": ("flop", 2.0 * T * FF * D),
        "attention": ("flop", 4.0 * H * DH * S * float(np.sum(lens))),
        "layernorm": ("bytes", T * D * (2 + 2) + 2 * D * 4),
        "embed_ln": ("bytes", T * (16 + 4 * D + 2 * D) + (S + BERT_TV) * 4 * D),
        "pooler": ("flop", 2.0 * B * D * D),
    }


def cpu_bert_rate(S: int, length: int):
    """The oracle's BERT encoder on one sequence of S positions (first `length` valid); returns
    (positions/s, seconds, cores)."""
    O = _oracle()
    O.build()
    O.set_loop_threads(1)
    shape = O.BERT_BASE
    blob = O.bert_seeded_blob(shape, SEED, 0)
    ids = O.token_ids(1, S, SEED, shape.vocab_size, stream=O.BERT_IDS_STREAM)
    mask = (np.arange(S)[None, :] < length).astype(np.int64)
    t0 = time.perf_counter()
    O.bert_forward(shape, blob, ids, None, mask)
    dt = time.perf_counter() - t0
    return S / dt, dt, os.cpu_count() or 1


def cpu_reference_rate(S: int, n_seq: int = 1, fp8: bool = False, repeats: int = 0):
    """The oracle (the reference's CPU lowering restated in C: OpenBLAS sgemm for the 2-D
    matmuls on all cores, single-threaded loop nests for the rest) on n_seq sequences of S
    tokens of the workload, repeated until about a second has passed when the forward is short
    (repeats = 0) or `repeats` times; returns (tokens/s, seconds of the forwards, cores)."""
    O = _oracle()
    O.build()
    O.set_loop_threads(1)
    shape = O.ModelShape(n_layer=L, n_embd=D, n_head=H, n_inner=FF)
    blob = O.seeded_blob(shape, SEED, 0)
    if fp8:
        blob = O.fp8_dequantized_blob(shape, blob)
    ids = O.token_ids(64, S, SEED, shape.vocab_size)[:n_seq]
    out = np.empty((n_seq, S, shape.vocab_size), dtype=np.float32)
    n, dt = 0, 0.0
    while (repeats and n < repeats) or (not repeats and (n == 0 or dt < 1.0)):
        t0 = time.perf_counter()
        O.forward(shape, blob, ids, out=out)
        dt += time.perf_counter() - t0
        n += 1
    return n * n_seq * S / dt, dt, os.cpu_count() or 1


def run_reference(args, rank, world):
    if rank != 0:
        return
    S = args.seq
    rates = []
    med = int(np.median(bert_lengths(args.batch, S))) if args.config == 3 else S
    for i in range(args.warmup + args.steps):
        if args.config == 3:
            r, dt, cores = cpu_bert_rate(S, med)
        else:
            r, dt, cores = cpu_reference_rate(S, fp8=args.config == 4, repeats=1)
        if i >= args.warmup:
            rates.append((r, dt))
    total_tokens = S * len(rates)
    total_s = sum(dt for _, dt in rates)
    value = total_tokens / total_s
    O = _oracle()
    line = {
        "impl": "reference",
        "metric": METRICS.get(args.config, "GPT-2 prefill tokens/s"),
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total_s / len(rates), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox weights N(0,0.02), uniform ids)",
        "config": {"workload": CONFIGS[args.config][0], "global_batch": args.batch, "seq_len": S,
                   "sample_per_step": f"1 sequence x {S} tokens"
                   + (f" ({med} valid, the median length)" if args.config == 3 else "")},
        # One sequence of the batch is timed per step and the rate is quoted per token: the full
        # batch's time is extrapolated from it (sequences are independent and equally long).
        "extrapolated": args.batch > 1,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "extrapolated": args.batch > 1,
                         "sample": f"1 x {S} tokens per step of the {args.batch}-sequence workload, extrapolated "
                                   f"per token; OpenBLAS sgemm ({O.blas_name().split('/')[-1]}) on "
                                   f"all {cores} cores, loop nests single-threaded as the reference's CPU lowering"
                                   + (" (BERT-base encoder)" if args.config == 3 else "")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_bert(args, rank, world, local_rank, pkg, torch, dist):
    """--config 3: the BERT-base BF16 encoder over this rank's shard of B128 x S512 right-padded
    sequences (device-resident ids, token types and mask; FP32 hidden states and pooled output
    written to HBM each step)."""
    Bm = pkg.bert
    row0, row1 = shard_rows(args.batch, world, rank)
    B, S = row1 - row0, args.seq
    T = B * S
    O = _oracle()
    lens_all = bert_lengths(args.batch, S)
    lens = lens_all[row0:row1]
    ids_h = np.ascontiguousarray(O.token_ids(args.batch, S, SEED, BERT_V, stream=O.BERT_IDS_STREAM)[row0:row1])
    mask_h = (np.arange(S)[None, :] < lens[:, None]).astype(np.int64)
    tt_h = np.zeros_like(ids_h)
    for b, n in enumerate(lens):  # second segment: the back half of the valid positions
        tt_h[b, n // 2:n] = 1
    Bm.init(Bm.BertConfig(L, D, H, FF, BERT_V, BERT_P, 1e-12, BERT_TV, 1), local_rank)
    Bm.init_seeded(SEED, 0)
    ids, tt, mask = (torch.from_numpy(a).cuda() for a in (ids_h, tt_h, mask_h))
    hidden = torch.empty(T, D, device="cuda", dtype=torch.float32)
    pooled = torch.empty(B, D, device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    def step():
        Bm.forward_device(ids.data_ptr(), tt.data_ptr(), None, mask.data_ptr(), B, S, hidden.data_ptr(),
                          pooled.data_ptr(), sp)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if Bm.status() != 0:
        raise SystemExit("device status word set during warm-up")
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    t_max = max_over_ranks(ev0.elapsed_time(ev1) / 1000.0, dist, "cuda")
    value = args.batch * S * args.steps / t_max

    Bm.profile_begin()
    nprof = 2
    for _ in range(nprof):
        step()
    prof = Bm.profile_end()
    torch.cuda.synchronize()
    work = bert_kernel_work(B, S, lens)
    kernels, roof = kernel_breakdown(prof, work, nprof, _peaks(), 3, T)
    ws = bert_kernel_work(args.batch, S, lens_all)
    total_flop = (ws["gemm_qkv"][1] + ws["gemm_attn_out"][1] + ws["gemm_intermediate"][1] + ws["gemm_output"][1]
                  + ws["attention"][1]) * L + ws["pooler"][1]

    e2e = None
    if args.e2e_steps > 0:
        pins = [torch.from_numpy(a).pin_memory() for a in (ids_h, tt_h, mask_h)]
        h_out = torch.empty((B, S, D), dtype=torch.float32).pin_memory()
        p_out = torch.empty((B, D), dtype=torch.float32).pin_memory()
        lib = Bm.lib()
        ptrs = [t.data_ptr() for t in pins]
        rc = lib.bert_forward_host(ptrs[0], ptrs[1], None, ptrs[2], B, S, h_out.data_ptr(), p_out.data_ptr())
        if rc != 0:
            raise SystemExit("bert_forward_host failed: " + Bm.last_error())
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            lib.bert_forward_host(ptrs[0], ptrs[1], None, ptrs[2], B, S, h_out.data_ptr(), p_out.data_ptr())
        et = time.perf_counter() - t0
        e2e = {"value": args.batch * S * args.e2e_steps / max_over_ranks(et, dist, "cuda"), "unit": "tokens/s",
               "h2d_bytes_per_step": int(sum(t.numel() * 8 for t in pins) * world),
               "d2h_bytes_per_step": int((h_out.numel() + p_out.numel()) * 4 * world), "steps": args.e2e_steps,
               "api": "bert_forward_host (C ABI, host buffers, synchronous)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        med = int(np.median(lens_all))
        r, dt, cores = cpu_bert_rate(S, med)
        cpu = {"value": r, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"1 sequence x {S} positions, {med} valid (the median length) ({dt:.1f} s); OpenBLAS "
                         f"sgemm ({O.blas_name().split('/')[-1]}) on all {cores} cores, loop nests single-threaded"}

    clocks = clk.summary()
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRICS[3], "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * t_max / args.steps, "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Philox weights N(0,0.02), LN gain 1, biases 0; uniform ids; seeded lengths)",
            "config": {"workload": f"{CONFIGS[3][0]}; FP32 hidden + pooled resident per shard",
                       "global_batch": args.batch, "seq_len": S, "per_rank_batch": B,
                       "valid_tokens": int(np.sum(lens_all)), "mean_length": float(np.mean(lens_all)),
                       "parallelism": f"batch-sharded dp{world}",
                       "l2": "no flush: every step moves > 2 GB of activations"},
            "valid_tokens_per_s": float(np.sum(lens_all)) * args.steps / t_max,
            "forward_tflops": total_flop / (t_max / args.steps) / 1e12,
            "roofline": roof, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": Bm.forward_launches(True, True) * args.steps,
        }
        print(json.dumps(line), flush=True)
    Bm.shutdown()
    if world > 1:
        dist.destroy_process_group()


def timed_steps(step, steps, stream, torch, dist, world):
    """Runs `steps` calls of step() between CUDA events on `stream` (barrier and synchronize on
    both sides); returns the max-over-ranks seconds."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return max_over_ranks(e0.elapsed_time(e1) / 1000.0, dist, "cuda")


def e2e_decoder(pkg, ids_h, steps, dist, world):
    """End to end through the drop-in symbol itself, called exactly as the reference's host program
    calls it (src/gpt/gpt2_call.cpp:62-68, :93-94): decomposed int64 memrefs of host ids and an
    all-ones mask in, a malloc'd FP32 logits memref out, read and freed by the caller every step.
    Host wall clock (the call is synchronous), max over ranks.  Returns (seconds per step, one
    result's checksum of its first and last logit rows)."""
    import ctypes
    P = ctypes.POINTER(ctypes.c_int64)
    B, S = ids_h.shape
    ids = np.ascontiguousarray(ids_h)
    mask = np.ones_like(ids)
    ip, mp = ids.ctypes.data_as(P), mask.ctypes.data_as(P)
    lib = pkg.lib()

    def call():
        m = lib.gpt2_decoder(ip, ip, 0, B, S, S, 1, mp, mp, 0, B, S, S, 1)
        if not m.allocated:
            raise SystemExit("gpt2_decoder failed: " + pkg.last_error())
        n = m.sizes[0] * m.sizes[1] * m.sizes[2]
        view = np.ctypeslib.as_array(m.aligned, shape=(n,))
        chk = float(view[:V].sum() + view[n - V:].sum())  # the caller reads its result
        pkg._libc.free(ctypes.cast(m.allocated, ctypes.c_void_p))
        return chk

    chk = call()  # warm-up: staging buffers, graph capture
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    et = time.perf_counter() - t0
    return max_over_ranks(et, dist, "cuda") / steps, chk


def e2e_pinned(pkg, ids_h, steps, dist, world):
    """The companion host-buffer entry point gpt2_forward_host with pinned ids and logits (one DMA
    each way, no staging); host wall clock, max over ranks.  Returns seconds per step."""
    import ctypes
    import torch
    B, S = ids_h.shape
    host_ids = torch.from_numpy(np.ascontiguousarray(ids_h)).pin_memory()
    host_logits = torch.empty((B, S, V), dtype=torch.float32, pin_memory=True)
    P = ctypes.POINTER
    ip = host_ids.numpy().ctypes.data_as(P(ctypes.c_int64))
    op = host_logits.numpy().ctypes.data_as(P(ctypes.c_float))
    lib = pkg.lib()
    if lib.gpt2_forward_host(ip, None, B, S, op) != 0:
        raise SystemExit("gpt2_forward_host failed: " + pkg.last_error())
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        lib.gpt2_forward_host(ip, None, B, S, op)
    et = time.perf_counter() - t0
    del host_logits
    return max_over_ranks(et, dist, "cuda") / steps


def forward_plus_gather(pkg, torch, dist, rank, world, ids, Bg, S, stream, logits_dtype, chunks, steps, warmup):
    """One step = this rank's forward and the gather of every shard's logits into rank 0's
    [Bg x S, LD_LOGITS] buffer, timed together (CUDA events on the compute stream, max over ranks).
    The shard runs as `chunks` sub-batches; a shard's chunk goes to rank 0 (NCCL send on a
    separate stream) as soon as its lm_head has written it, while the next chunk computes.  Rank 0
    writes its own shard in place and posts every receive up front.  Returns seconds per step."""
    B = ids.shape[0]
    if B % chunks:
        chunks = 1
    bc = B // chunks
    tdt = torch.float32 if logits_dtype == pkg.DTYPE_F32 else torch.bfloat16
    if rank == 0:
        full = torch.empty(Bg * S, LD_LOGITS, device="cuda", dtype=tdt)
        outs = [full[k * bc * S:(k + 1) * bc * S] for k in range(chunks)]
    else:
        local = torch.empty(B * S, LD_LOGITS, device="cuda", dtype=tdt)
        outs = [local[k * bc * S:(k + 1) * bc * S] for k in range(chunks)]
    ids_k = [ids[k * bc:(k + 1) * bc] for k in range(chunks)]
    comm = torch.cuda.Stream()
    evs = [torch.cuda.Event() for _ in range(chunks)]

    def step():
        reqs = []
        if rank == 0:
            ops = [dist.P2POp(dist.irecv, full[(p * B + k * bc) * S:(p * B + (k + 1) * bc) * S], p)
                   for p in range(1, world) for k in range(chunks)]
            reqs = dist.batch_isend_irecv(ops)
        for k in range(chunks):
            pkg.forward_device(ids_k[k].data_ptr(), None, bc, S, outs[k].data_ptr(), LD_LOGITS, stream.cuda_stream,
                               logits_dtype)
            if rank != 0:
                evs[k].record(stream)
                with torch.cuda.stream(comm):
                    comm.wait_event(evs[k])
                    # the same batched point-to-point API as rank 0's receives (one communicator for both)
                    for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, outs[k], 0)]):
                        r.wait()
        for r in reqs:
            r.wait()
        stream.wait_stream(comm)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
        t = timed_steps(step, steps, stream, torch, dist, world)
    del outs
    return t / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS),
                    help="reference configuration (2 = the headline BF16 workload)")
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch (sequences); default: the config's batch in total (strong scaling) or "
                         "per rank (weak)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong (default): the configuration's batch split over the ranks, as the "
                         "configuration states it; weak: every rank runs the configuration's batch")
    ap.add_argument("--seq", type=int, default=None, help="default: the config's")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--gather-steps", type=int, default=5)
    ap.add_argument("--gather-chunks", type=int, default=2,
                    help="sub-batches per shard in the forward + gather step (1 = gather after the forward)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true", help="skip the forward + logits gather step (N > 1)")
    ap.add_argument("--no-decode", action="store_true", help="skip the KV-cache decode measurement")
    args = ap.parse_args()

    global L, D, H, FF
    wl_name, L, D, H, FF, dtype_code, dtype_label, gb, gs = CONFIGS[args.config]
    if args.batch is None:
        args.batch = gb * (int(os.environ.get("WORLD_SIZE", "1")) if args.scaling == "weak" else 1)
    if args.seq is None:
        args.seq = gs
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    pkg = _pkg()
    if args.config == 3:
        run_bert(args, rank, world, local_rank, pkg, torch, dist)
        return
    row0, row1 = shard_rows(args.batch, world, rank)
    B, S = row1 - row0, args.seq
    T = B * S

    pkg.init(pkg.Gpt2Config(L, D, H, FF, V, 1024, 1e-5, dtype_code), local_rank)
    pkg.init_seeded(SEED, 0)
    ids_all = pkg.seeded_ids(args.batch, S, SEED, V)
    ids_h = np.ascontiguousarray(ids_all[row0:row1])
    ids = torch.from_numpy(ids_h).cuda()
    logits = torch.empty(T, LD_LOGITS, device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    def step():
        pkg.forward_device(ids.data_ptr(), None, B, S, logits.data_ptr(), LD_LOGITS, sp)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if pkg.status() != 0:
        raise SystemExit("device status word set during warm-up")
    with ClockSampler(local_rank) as clk:
        t_max = timed_steps(step, args.steps, stream, torch, dist, world)
    value = args.batch * S * args.steps / t_max
    step_ms = 1000.0 * t_max / args.steps

    # Per-kernel breakdown (separate, profiled steps of the same workload: an event pair around
    # every launch).  The profiled step runs at higher clocks than the timed one (the timed
    # step is power-capped), so each kernel's time is also given scaled to the timed step by its
    # share, and the roofline is computed from that scaled time.
    pkg.profile_begin()
    nprof = 2
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(nprof):
        step()
    p1.record(stream)
    prof = pkg.profile_end()
    torch.cuda.synchronize()
    profiled_step_ms = p0.elapsed_time(p1) / nprof
    work = kernel_work(B, S, args.config)
    ffma = pkg.k_ffma_peak() if args.config == 1 else None
    kernels, roof = kernel_breakdown(prof, work, nprof, _peaks(), args.config, T, ffma, timed_step_ms=step_ms)
    fl = kernel_work(B, S)
    total_flop = (fl["gemm_qkv"][1] + fl["gemm_proj"][1] + fl["gemm_fc"][1] + fl["gemm_mproj"][1]) * L \
        + fl["lm_head"][1] + fl["attention"][1] * L
    fwd_tflops = total_flop / (t_max / args.steps) / 1e12

    # The same forward with bf16 logits (the optional store of the lm_head epilogue): half the
    # bytes written; reported beside the FP32 headline.
    bf16_logits = None
    if dtype_code >= 1:
        lg16 = torch.empty(T, LD_LOGITS, device="cuda", dtype=torch.bfloat16)

        def step16():
            pkg.forward_device(ids.data_ptr(), None, B, S, lg16.data_ptr(), LD_LOGITS, sp, pkg.DTYPE_BF16)
        for _ in range(3):
            step16()
        n16 = max(3, args.steps // 2)
        t16 = timed_steps(step16, n16, stream, torch, dist, world)
        pkg.profile_begin()
        step16()
        prof16 = pkg.profile_end()
        torch.cuda.synchronize()
        head_ms, _ = prof16["lm_head"]
        bf16_logits = {"tokens_per_s": args.batch * S * n16 / t16, "ms_per_step": 1000.0 * t16 / n16,
                       "lm_head_ms_profiled": head_ms, "steps": n16,
                       "logits_bytes_per_rank": int(T * V * 2)}
        del lg16

    # Forward + gather of every shard's logits into rank 0 (NCCL over NVLink), FP32 and bf16.
    gather = None
    if world > 1 and not args.no_gather:
        del logits
        gather = {"method": f"NCCL send/recv into one [global batch x S, {LD_LOGITS}] buffer on rank 0; "
                            "each shard in sub-batches, a sub-batch sent as soon as its lm_head is done"}
        for lab, dt in (("f32", pkg.DTYPE_F32), ("bf16", pkg.DTYPE_BF16)):
            if dt == pkg.DTYPE_BF16 and dtype_code == 0:
                continue
            for ch in sorted({1, args.gather_chunks}):
                ts = forward_plus_gather(pkg, torch, dist, rank, world, ids, args.batch, S, stream, dt, ch,
                                         args.gather_steps, 2)
                gather[f"{lab}_chunks{ch}"] = {
                    "ms_per_step": 1000.0 * ts, "tokens_per_s_forward_plus_gather": args.batch * S / ts,
                    "bytes_to_rank0": int((args.batch - B) * S * V * (4 if dt == pkg.DTYPE_F32 else 2))}
        best = max((v for k, v in gather.items() if k.startswith("f32_")),
                   key=lambda v: v["tokens_per_s_forward_plus_gather"])
        gather["tokens_per_s_forward_plus_gather"] = best["tokens_per_s_forward_plus_gather"]
        logits = torch.empty(T, LD_LOGITS, device="cuda", dtype=torch.float32)

    # End to end: through the drop-in gpt2_decoder (malloc'd result, as the reference's host program
    # receives it) and through gpt2_forward_host with pinned buffers.  Host memory for the results
    # is bounded by half of what is free, shared by this host's ranks; with little memory the
    # end-to-end steps use fewer sequences per rank and say so.
    e2e = None
    if args.e2e_steps > 0:
        import psutil
        local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
        avail = psutil.virtual_memory().available
        eB = max(1, min(B, int(avail // 2 // (2 * S * V * 4 * local_ranks))))
        eBt = torch.tensor([eB], device="cuda")
        if world > 1:
            dist.all_reduce(eBt, op=dist.ReduceOp.MIN)  # the same work on every rank
        eB = int(eBt.item())
        sub = ids_h[:eB]
        t_dec, _ = e2e_decoder(pkg, sub, args.e2e_steps, dist, world)
        t_pin = e2e_pinned(pkg, sub, args.e2e_steps, dist, world)
        h2d = int(sub.nbytes * 2 * world)  # ids and the all-ones mask
        d2h = int(eB * S * V * 4 * world)
        e2e = {"value": eB * world * S / t_dec, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": args.e2e_steps, "per_rank_batch": eB,
               "api": "gpt2_decoder (the drop-in symbol; decomposed memrefs, malloc'd FP32 result freed by the "
                      "caller each step)",
               "d2h_gbs": d2h / t_dec / 1e9,
               "pinned": {"value": eB * world * S / t_pin, "unit": "tokens/s", "d2h_gbs": d2h / t_pin / 1e9,
                          "api": "gpt2_forward_host (pinned host ids and logits)"},
               "decoder_vs_pinned": t_pin / t_dec}

    # Incremental decoding on the same model (reported beside the prefill number): greedy
    # generation with the KV cache, 64 new tokens after a 128-token prompt, per-token time from the
    # difference between 64 and 1 generated tokens.
    decode = None
    if args.config in (1, 2) and world == 1 and not args.no_decode:
        decode = {}
        for db in (1, 16):
            prompt = pkg.seeded_ids(db, 128, SEED, V)

            def gen(k):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                pkg.generate(prompt, k)
                return time.perf_counter() - t0
            gen(64)
            t1 = min(gen(1) for _ in range(3))
            tn = min(gen(64) for _ in range(3))
            dstep = (tn - t1) / 63
            decode[f"B{db}"] = {"ms_per_token_step": 1e3 * dstep, "tokens_per_s": db / dstep, "prompt": 128,
                                "new_tokens": 64}
        decode["api"] = "gpt2_generate (KV cache, one CUDA graph per step)"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, dt, cores = cpu_reference_rate(S, fp8=args.config == 4)
        O = _oracle()
        cpu = {"value": r, "unit": "tokens/s", "cores": cores, "kind": "port", "extrapolated": args.batch > 1,
               "sample": f"1 sequence x {S} tokens ({dt:.1f} s{', repeated' if dt * r > 1.5 * S else ''}) of the "
                         f"{args.batch}-sequence workload; OpenBLAS sgemm ({O.blas_name().split('/')[-1]}) on all "
                         f"{cores} cores, loop nests single-threaded"}

    clocks = clk.summary()
    weight_bytes = (L * (12 * D * D + 13 * D) + (V + 1024) * D) * (4 if dtype_code == 0 else 2)
    moved_gb = (weight_bytes + T * V * 4) / 1e9
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRICS.get(args.config, "GPT-2 prefill tokens/s"),
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": value / PUBLISHED_B1S5_TOKENS_PER_S if args.config == 0 else None,
            "dtype": dtype_label,
            "data": "synthetic (seeded Philox weights N(0,0.02), LN gain 1, biases 0; uniform token ids)",
            "config": {"workload": f"{wl_name} with global batch {args.batch} x {S}, logits FP32 resident per shard",
                       "global_batch": args.batch, "seq_len": S, "per_rank_batch": B,
                       "parallelism": f"batch-sharded dp{world} ({args.scaling} scaling)",
                       "l2": f"no flush: every step moves > {moved_gb:.2f} GB (weights + FP32 logits), "
                             "more than the 126 MB L2"},
            "forward_tflops": fwd_tflops,
            "profiled_step_ms": profiled_step_ms,
            "roofline": roof,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "bf16_logits": bf16_logits,
            "logits_gather": gather,
            "decode": decode,
            "clocks": clocks,
            "gpu_launches": pkg.forward_launches(B, S, False) * args.steps,
        }
        print(json.dumps(line), flush=True)
    pkg.shutdown()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
