#!/usr/bin/env python3
"""Training-step benchmark: GPT-2-small shape, train tokens/sec, MFU vs the measured bf16 peak.

Workload (one step): 8 sequences x 1024 tokens per GPU of a 12-layer, n_embd 768, 12-head,
GELU-FFN 3072, LayerNorm, learned positions, tied-embedding GPT with vocab 50257; seeded
synthetic Zipf(1.1) token ids; forward -> cross-entropy -> backward -> clip -> AdamW
(lr 3e-4, betas 0.9/0.95, wd 0.1). Data parallel over N GPUs (one process per GPU, NCCL
gradient all-reduce), weak scaling (8 sequences per GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is the whole-job tokens/s with the token batches already resident in HBM
(llmgpu_train_step_device); `e2e` is the same step through the public C ABI with host
token buffers (host->device copy of the tokens and device->host read of loss/grad-norm
inside every timed step). Timing: CUDA events on the library's stream, barrier +
synchronize on both sides, max over ranks. The per-step working set (logits alone are
0.82 GB) is far larger than the 126 MB L2, so no explicit L2 flush is needed.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-cpp_b200", "python"))

CFG = dict(vocab_size=50257, n_layers=12, n_heads=12, n_embd=768, block_size=1024,
           weight_tying=True)
B, T = 8, 1024
HP = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)
REF_T = 16          # tokens of the bounded CPU-reference sample (one sequence)
# DRAM bytes read + written per GEMM launch of the GPT-2-small step, averaged over its 98
# launches: one ncu capture of those launches (dram__bytes_read.sum + dram__bytes_write.sum,
# cold caches) of `bench.py --steps 1 --warmup 1 --no-cpu-baseline`
GEMM_TRAFFIC_BYTES = 107.6e6


def algorithmic_flops_per_token(cfg=CFG, T=T):
    """F_tok = 6*N_mm + 6*L*T*C (causal attention counted once; recompute not counted).
    N_mm counts matmul weights incl. the lm head (tied or not), not the embeddings."""
    C, L, V = cfg["n_embd"], cfg["n_layers"], cfg["vocab_size"]
    F = 4 * C
    n_mm = L * (4 * C * C + 2 * C * F) + C * V
    return 6 * n_mm + 6 * L * T * C, n_mm


# The other configurations of the path, for `--config` (the default line is GPT-2-small):
# model config, sequences per GPU, sequence length, workload text.
OTHER_CONFIGS = {
    "tiny": (dict(vocab_size=256, n_layers=4, n_heads=4, n_embd=128, block_size=128), 8, 128,
             "tiny char-level GPT (4L, n_embd 128, 4 heads, GELU FFN 512, vocab 256), seq 128, 8 seq/GPU"),
    "llama": (dict(vocab_size=32000, n_layers=24, n_heads=16, n_embd=1024, block_size=2048,
                   weight_tying=False, use_rmsnorm=True, ffn_swiglu=True, ffn_hidden=2816,
                   rope_qk=True), 4, 2048,
              "Llama-style (24L, n_embd 1024, 16 heads, SwiGLU 2816, RoPE on Q/K, RMSNorm, untied, "
              "vocab 32000), seq 2048, 4 seq/GPU"),
    "mamba": (dict(vocab_size=32000, n_layers=12, n_heads=1, n_embd=768, block_size=2048,
                   use_rmsnorm=True, use_mamba=True, d_inner=1536, d_state=16, dt_rank=48,
                   conv_kernel=4), 4, 2048,
              "Mamba (12 blocks, E 768, D 1536, N 16, R 48, K 4, RMSNorm, tied, vocab 32000), "
              "seq 2048, 4 seq/GPU"),
    "moe": (dict(vocab_size=32000, n_layers=12, n_heads=12, n_embd=768, block_size=1024,
                 moe_experts=8, moe_top_k=2, moe_aux_coef=0.01), 8, 1024,
            "MoE (12L, n_embd 768, 12 heads, 8 GELU experts of 3072, top-2, aux 0.01, tied, "
            "vocab 32000), seq 1024, 8 seq/GPU"),
}


def flops_per_token(cfg, T):
    """F_tok = 6*N_mm + (attention) 6*L*T*C, with N_mm the matmul weights one token passes
    through (the active experts for MoE, the head counted even when tied)."""
    C, L, V = cfg["n_embd"], cfg["n_layers"], cfg["vocab_size"]
    if cfg.get("use_mamba"):
        D, N, R = cfg["d_inner"], cfg["d_state"], cfg["dt_rank"]
        n_mm = L * (2 * D * C + (R + 2 * N) * D + D * R + C * D) + C * V
        return 6 * n_mm, n_mm
    if cfg.get("moe_experts"):
        k = cfg.get("moe_top_k", 2)
        n_mm = L * (4 * C * C + k * 2 * C * 4 * C + C * cfg["moe_experts"]) + C * V
    elif cfg.get("ffn_swiglu"):
        n_mm = L * (4 * C * C + 3 * C * cfg["ffn_hidden"]) + C * V
    else:
        n_mm = L * (4 * C * C + 2 * C * 4 * C) + C * V
    return 6 * n_mm + 6 * L * T * C, n_mm


def zipf_tokens(vocab, n, seed, s=1.1):
    import numpy as np
    rng = np.random.default_rng(seed)
    pk = np.arange(1, vocab + 1, dtype=np.float64) ** (-s)
    pk /= pk.sum()
    return rng.choice(vocab, size=n, p=pk).astype(np.int32)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                "sw_power_cap"], f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ CPU baselines
def ref_binary():
    p = os.path.join(ROOT, "oracle", "_ref", "ref_step")
    return p if os.path.exists(p) else None


def run_reference_cpu(steps, T_sample, model_cfg=CFG, B_sample=1, warmup=0, seed=1234):
    """The unmodified reference train step (oracle/_ref/ref_step, built from the reference
    sources) on all host cores: warmup + steps optimizer steps of Trainer::train_step_accum
    over B_sample sequences of T_sample seeded Zipf(1.1) tokens, reference initialisation,
    constant LR. Returns (seconds of each timed step, threads)."""
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as td:
        env = dict(os.environ, OMP_NUM_THREADS=str(threads))
        args = [ref_binary(), "-", "-", str(B_sample), str(T_sample), td,
                f"steps={warmup + steps}", "timing_only=1", f"seed={seed}",
                f"vocab={model_cfg['vocab_size']}", f"layers={model_cfg['n_layers']}",
                f"heads={model_cfg['n_heads']}", f"embd={model_cfg['n_embd']}",
                f"block={model_cfg['block_size']}", f"tied={int(model_cfg.get('weight_tying', True))}"]
        args += [f"{k}={v}" for k, v in HP.items()]
        subprocess.run(args, check=True, env=env, stdout=subprocess.DEVNULL,
                       stderr=subprocess.DEVNULL)
        with open(os.path.join(td, "timing.txt")) as f:
            times = [float(x) for x in f.read().split()]
    return times[warmup:], threads


# ------------------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    line = {"impl": "reference", "metric": "train_tokens_per_sec", "unit": "tokens/s",
            "higher_is_better": True, "n_gpus": args.gpus, "data": "synthetic",
            "dtype": "f32", "config": workload_config(args.gpus)}
    if ref_binary() is None:
        line["unavailable"] = "oracle/_ref/ref_step not built (needs the reference sources)"
        print(json.dumps(line))
        return 0
    # One reference optimizer step over a single 16-token sequence of this model takes about
    # 30 s on the host cores (a single-threaded lm-head backward over V=50257, three forward
    # recomputes and an AdamW loop over 124M parameters): one warm-up step, then the median
    # of at most three timed steps, so that the arm ends within a few minutes.
    warm = min(args.warmup, 1)
    steps = max(1, min(args.steps, 3))
    times, threads = run_reference_cpu(steps, REF_T, warmup=warm)
    per = statistics.median(times)
    value = REF_T / per
    sample = (f"{warm} warm-up + median of {steps} reference optimizer step(s) "
              f"(Trainer::train_step_accum), each over 1 sequence of {REF_T} Zipf tokens of the "
              f"full 12-layer/768/50257 model; {per:.1f} s per step")
    line.update({"value": value, "steps": steps, "warmup": warm, "ms_per_step": per * 1e3,
                 "scaling": "weak", "vs_baseline": None,
                 "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                                  "kind": "reference", "sample": sample},
                 "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    print(json.dumps(line))
    return 0


def workload_config(n):
    return {"workload": "GPT-2-small train step (12L, n_embd 768, 12 heads, GELU FFN 3072, "
                        "LayerNorm, learned pos, tied, vocab 50257), seq 1024, 8 seq/GPU",
            "global_batch": 8 * n, "seq_len": T, "parallelism": f"dp{n}",
            "tokens": "Zipf(1.1) synthetic ids, seeded",
            "l2": "no flush: per-step working set (0.82 GB logits + 1.1 GB weights/state) >> L2"}


# ------------------------------------------------------------------------------ our arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="sequences per GPU (0: the workload's own); smaller cases for profiling")
    ap.add_argument("--config", default="gpt2-small", choices=["gpt2-small"] + sorted(OTHER_CONFIGS),
                    help="workload (the headline line is gpt2-small)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import numpy as np
    import torch
    torch.cuda.set_device(local)
    dist = None
    uid = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        from llmgpu.trainer import unique_id
        obj = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    from llmgpu.trainer import Trainer, make_config
    model_cfg, B, T, workload = (CFG, globals()["B"], globals()["T"], None)
    if args.config != "gpt2-small":
        model_cfg, B, T, workload = OTHER_CONFIGS[args.config]
    if args.batch > 0:
        B = args.batch
        workload = (workload or workload_config(1)["workload"]).replace("8 seq/GPU", "") + \
            f" [profiling case: {B} seq/GPU]"
    cfg = make_config(**model_cfg)
    tr = Trainer(cfg, B, T, rank=rank, world=world, uid=uid)
    tr.set_adamw(**HP)
    tr.set_train(grad_clip=1.0)
    K, W = args.steps, args.warmup
    toks = zipf_tokens(model_cfg["vocab_size"], (W + 2 * K) * B * T, 1234 + rank).reshape(-1, B, T)
    stream = torch.cuda.ExternalStream(tr.stream())

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def maxed(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(W):
        tr.train_step(toks[i])
    # ---------------- value: tokens resident in HBM
    dev_toks = torch.from_numpy(toks[W:W + K].copy()).to(f"cuda:{local}")
    step_bytes = B * T * 4
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches = 0
    for i in range(K):
        tr.train_step_device(dev_toks[i].data_ptr(), B, T)
        launches += tr.last_launches()
    e1.record(stream)
    barrier()
    ms_dev = e0.elapsed_time(e1) / K
    # ---------------- e2e: host tokens through the public C ABI
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    losses = []
    for i in range(K):
        loss, gn, _ = tr.train_step(toks[W + K + i])
        losses.append(loss)
    e3.record(stream)
    barrier()
    clocks = sampler.stop()
    ms_e2e = e2.elapsed_time(e3) / K
    ms_dev, ms_e2e = maxed(ms_dev), maxed(ms_e2e)
    timings = tr.last_timings()
    # ---------------- GEMM roofline: the same steps with every tcgen05 GEMM launch bracketed
    # by CUDA events on the library stream (eager execution; not part of `value`)
    tr.set_profile(True)
    tr.gemm_stats(reset=True)
    for i in range(K):
        tr.train_step_device(dev_toks[i].data_ptr(), B, T)
    barrier()
    gflops, gms, glaunch = tr.gemm_stats(reset=True)
    tr.set_profile(False)

    peak, peak_sus, hbm, peak_kind = peaks()
    f_tok, n_mm = flops_per_token(model_cfg, T)
    tokens_step = world * B * T
    value = tokens_step / (ms_dev / 1e3)
    e2e = tokens_step / (ms_e2e / 1e3)
    mfu = f_tok * value / (world * peak * 1e12)
    gemm_tflops = gflops / (gms / 1e3) / 1e12 if gms > 0 else 0.0
    if rank == 0:
        line = {
            "metric": "train_tokens_per_sec", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_dev,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world) if workload is None else
                      {"workload": workload, "global_batch": B * world, "seq_len": T,
                       "parallelism": f"dp{world}", "tokens": "Zipf(1.1) synthetic ids, seeded"},
            "mfu": {"value": mfu, "peak_tflops": peak, "peak": peak_kind,
                    "flops_per_token": f_tok, "n_mm": n_mm},
            "e2e": {"value": e2e, "unit": "tokens/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": step_bytes, "d2h_bytes_per_step": 32},
            "gpu_launches": launches,
            "roofline": {"kernel": "tcgen05 GEMMs (gemm_bf16_pair_kernel, gemm_bf16_tc_kernel): "
                                   "every GEMM launch of the step",
                         "bound": "tensor", "achieved": gemm_tflops, "peak": peak_sus,
                         "unit": "TFLOP/s", "frac": gemm_tflops / peak_sus,
                         "peak_kind": f"{peak_kind} sustained bf16 (kernel timed inside a long step)",
                         "traffic": GEMM_TRAFFIC_BYTES if workload is None else None,
                         "traffic_unit": "DRAM bytes read + written per GEMM launch, averaged "
                                         "over the step's launches (one ncu capture, cold caches)",
                         "launches_per_step": glaunch / max(K, 1),
                         "gemm_ms_per_step": gms / max(K, 1),
                         "flops_per_step": gflops / max(K, 1)},
            "phase_ms": timings,
            "clocks": clocks,
            "loss_last": losses[-1],
        }
        if world == 1 and not args.no_cpu_baseline and ref_binary() is not None and \
                (workload is None or args.config == "tiny"):
            try:
                if workload is None:
                    # GPT-2-small: one optimizer step over one 16-token sequence (~30 s)
                    times, threads = run_reference_cpu(1, REF_T)
                    secs = times[0]
                    line["cpu_baseline"] = {
                        "value": REF_T / secs, "unit": "tokens/s", "cores": threads,
                        "kind": "reference",
                        "sample": f"the unmodified reference (oracle/_ref/ref_step) training "
                                  f"one sequence of {REF_T} tokens of the same model for one "
                                  f"optimizer step ({secs:.1f} s)"}
                else:
                    # the tiny configuration in full: 8 sequences of 128 tokens per step
                    times, threads = run_reference_cpu(3, T, model_cfg, B_sample=B, warmup=1)
                    secs = statistics.median(times)
                    line["cpu_baseline"] = {
                        "value": B * T / secs, "unit": "tokens/s", "cores": threads,
                        "kind": "reference",
                        "sample": f"the unmodified reference (oracle/_ref/ref_step): the whole "
                                  f"step of {B} x {T} tokens, one warm-up and the median of 3 "
                                  f"steps ({secs:.2f} s per step)"}
            except Exception as ex:  # the baseline is reported, never fatal
                line["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
        print(json.dumps(line), flush=True)
    tr.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
