"""Decode benchmark: ForgeLM's token loop on B200 through libforge_b200.so.

Workloads (synthetic seeded weights and prompts):
  c2 (default): Forge-98M fp32, batch 1 per GPU, prompt 64 uniform-random
      ids, 512 new tokens at temperature 0.7, top-k 30, repetition penalty
      1.1, no-repeat-ngram 4, RNG seed 1 (+rank).  One step = one full
      generate (prefill + 512 sampled tokens).
  c3: Forge-98M fp32, 64 sequences split evenly over the GPUs, prompts of
      256 ids, 768 greedy tokens.  One step = one generate of the shard.
  c4: forge-220m fp32, 16 sequences split over the GPUs, prompts of 1024 ids
      (the full context), sampled at T 0.7, top-k 30: every new token slides
      the window, so every step re-prefills all 1024 positions (tensor-core
      bound).  One bench step = 16 new tokens of the 512 the workload names
      (a bounded sample; each token costs the same full re-prefill).
  c5: Forge-98M with bf16 weights (FB2_WEIGHTS_BF16), 32 sequences per GPU
      (256 on 8 GPUs), prompt lengths uniform in [64, 960], greedy decode
      (the workload decodes every sequence to the 1024-token context; one
      bench step = 64 new tokens of that, a bounded sample).  KV-bound.
Metric: decode tokens/s, whole job (sum over GPUs), max over ranks of the
device time.  N>1: one process per GPU, independent sequences, no data-path
collective (weak scaling for c2, strong for c3).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3]
  python bench.py --impl reference ...   # the reference algorithm on CPU
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FORGE_98M = dict(vocab_size=16384, context_length=1024, d_model=768, n_layers=12, n_heads=12)
FORGE_220M = dict(vocab_size=16384, context_length=1024, d_model=1024, n_layers=16, n_heads=16)
# Measured DRAM traffic of the dominant kernel is read from a record written
# by `bench.py --record-traffic <ncu csv>` (the one-pass launch-list capture
# with dram__bytes_read.sum and dram__bytes_write.sum); it is used only when
# the record names the source fingerprint the loaded library was built from
# (the build writes it beside the library), else null.
TRAFFIC_RECORD = os.path.join(ROOT, "profiles", "traffic_record.json")
WEIGHT_SEED = 1234

WORKLOADS = {
    "c2": dict(name="Forge-98M fp32 bs1: prompt 64, 512 sampled tokens (T 0.7, top-k 30, rep 1.1, ngram 4)",
               model=FORGE_98M, seqs_total=None, seqs_per_gpu=1, prompt_len=64, new_tokens=512,
               temperature=0.7, top_k=30, penalty=1.1, ngram=4, scaling="weak"),
    "c3": dict(name="Forge-98M fp32 bs64: prompts 256, 768 greedy tokens, sequences split over GPUs",
               model=FORGE_98M, seqs_total=64, seqs_per_gpu=None, prompt_len=256, new_tokens=768,
               temperature=0.0, top_k=0, penalty=1.0, ngram=0, scaling="strong"),
    "c5": dict(name="Forge-98M bf16 weights, 32 sequences per GPU, prompts U[64, 960], greedy; 64 new tokens per "
                    "bench step of the decode to the 1024-token context",
               model=FORGE_98M, seqs_total=None, seqs_per_gpu=32, prompt_len=(64, 960), new_tokens=64,
               temperature=0.0, top_k=0, penalty=1.0, ngram=0, scaling="weak", weight_dtype="bf16"),
    "c4": dict(name="forge-220m fp32 bs16: prompts 1024 (full context), sampled T 0.7 top-k 30; every token "
                    "re-prefills the 1024-token window; 16 of the 512 tokens per bench step",
               model=FORGE_220M, seqs_total=16, seqs_per_gpu=None, prompt_len=1024, new_tokens=16,
               temperature=0.7, top_k=30, penalty=1.0, ngram=0, scaling="strong", bound="tensor"),
}


def model_name(m: dict) -> str:
    name = "Forge-98M" if m == FORGE_98M else "forge-220m" if m == FORGE_220M else "custom"
    return (f"{name} (V {m['vocab_size']}, ctx {m['context_length']}, D {m['d_model']}, L {m['n_layers']}, "
            f"H {m['n_heads']})")


def flops_per_sequence_step(m: dict, T: int) -> float:
    """FLOPs of one full re-forward of a T-token window (the sliding-window
    step): the block projections for every row, causal attention (scores
    and context, T(T+1)/2 pairs each), and the head on the last row."""
    D, L, V = m["d_model"], m["n_layers"], m["vocab_size"]
    return 2.0 * T * L * 12 * D * D + 2.0 * L * T * (T + 1) * D + 2.0 * D * V


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--new-tokens", type=int, default=None, help="override the workload's new-token count "
                    "(smaller cases for profiling; the default is the workload's)")
    ap.add_argument("--skip-e2e", action="store_true", help="omit the host-buffer e2e leg (profiling runs)")
    ap.add_argument("--record-traffic", metavar="NCU_CSV", default=None,
                    help="write the DRAM traffic record of --workload from an ncu --csv capture and exit")
    ap.add_argument("--kernel-times", action="store_true",
                    help="after the warm-up, run one step under the CUDA activity profiler (CUPTI, through "
                         "torch.profiler) and print every kernel's warm device time instead of the bench line")
    ap.add_argument("--record-kernel", default="k_decode_mega")
    ap.add_argument("--record-steps-per-launch", type=int, default=511)
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, even split of `total` sequences: (first, count)."""
    per, extra = divmod(total, world)
    first = rank * per + min(rank, extra)
    return first, per + (1 if rank < extra else 0)


def prompts_for(first: int, count: int, plen, vocab: int) -> list[np.ndarray]:
    """Uniform-random prompt ids, seed 42 + global sequence index; `plen` is a
    length or a (lo, hi) range drawn per sequence from the same seed."""
    out = []
    for i in range(count):
        g = np.random.default_rng(42 + first + i)
        n = plen if isinstance(plen, int) else int(g.integers(plen[0], plen[1] + 1))
        out.append(g.integers(0, vocab, n).astype(np.int32))
    return out


def weight_bytes(m: dict, dtype: str = "fp32") -> float:
    """Bytes of every parameter one decode step streams once (shared by all
    sequences of the step): block weights and biases, ln_f, the tied head.
    bf16 narrows the projections and the head to 2 bytes."""
    D, L, V = m["d_model"], m["n_layers"], m["vocab_size"]
    wide = 2.0 if dtype == "bf16" else 4.0
    return wide * (L * 12 * D * D + V * D) + 4.0 * (L * 13 * D + 2 * D)


def sequence_bytes(m: dict, T: int) -> float:
    """Bytes one decode step moves per sequence whose attention spans T keys:
    its token and position rows and the K/V cache of T positions."""
    D, L = m["d_model"], m["n_layers"]
    return 4.0 * 2 * D + 4.0 * 2 * L * T * D


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def ref_flops_per_token(m: dict, T: int) -> float:
    """FLOPs of one reference step (GptModel.ForwardLast of a T-token window:
    every row through the blocks, full T x T attention scores and context
    before the causal mask, logits of every row, Sampler.cs:91-95)."""
    D, L, V = m["d_model"], m["n_layers"], m["vocab_size"]
    return 2.0 * T * (L * 12 * D * D + V * D) + 4.0 * L * T * T * D


CPU_SAMPLE_TOKENS = 40


def cpu_reference_sample(wl: dict, n_tokens: int = CPU_SAMPLE_TOKENS, full_run: bool = True) -> dict:
    """The reference algorithm (full re-forward of the window for every token,
    logits for every row; the oracle's restatement of CpuBackend + Sampler)
    on all host cores.  Measured: the first n_tokens of sequence 0 of the
    workload.  Those are the cheapest tokens of the run (the window grows),
    so with full_run the windows of the whole run are also sampled: one
    reference step is timed at five window lengths spread over the run, a
    cost model time(T) = a + b*flops(T) is fitted to them, and the run's
    rate is 'tokens / sum of the model over every step'."""
    from oracle import oracle as O
    O.set_threads(0)
    m = wl["model"]
    cfg = O.Config(m["vocab_size"], m["context_length"], m["d_model"], m["n_layers"], m["n_heads"])
    params = O.init_params(cfg, WEIGHT_SEED)
    if wl.get("weight_dtype") == "bf16":
        params = O.round_bf16(cfg, params)
    prompt = prompts_for(0, 1, wl["prompt_len"], m["vocab_size"])[0]
    n = max(1, min(wl["new_tokens"], n_tokens))
    t0 = time.perf_counter()
    ids = O.generate(cfg, params, prompt, n, wl["temperature"], wl["top_k"], O.DotNetRandom(1),
                     repetition_penalty=wl["penalty"], no_repeat_ngram=wl["ngram"])
    dt = time.perf_counter() - t0
    ctx = m["context_length"]
    out = {"value": len(ids) / dt, "unit": "tokens/s", "cores": O.get_threads(), "cpu_model": cpu_model(),
           "kind": "port",
           "sample": f"first {len(ids)} of {wl['new_tokens']} tokens of sequence 0 (prompt {len(prompt)}), full "
                     f"re-forward per token as the reference CPU backend does",
           "seconds": dt, "ids": ids}
    if full_run:
        steps_T = [min(len(prompt) + k, ctx) for k in range(wl["new_tokens"])]
        probe = sorted(set(int(x) for x in np.linspace(steps_T[0], steps_T[-1], 5)))
        rng = np.random.default_rng(0)
        secs = []
        for T in probe:
            w = rng.integers(0, m["vocab_size"], T).astype(np.int32)
            t0 = time.perf_counter()
            O.forward_last(cfg, params, w)
            secs.append(time.perf_counter() - t0)
        x = np.array([ref_flops_per_token(m, T) for T in probe])
        if len(probe) > 1:
            b, a = np.polyfit(x, np.array(secs), 1)
        else:
            a, b = 0.0, secs[0] / x[0]
        total = sum(a + b * ref_flops_per_token(m, T) for T in steps_T)
        out["full_run"] = {"value": wl["new_tokens"] / total, "unit": "tokens/s",
                           "method": f"one reference step timed at windows {probe}; time(T) = a + b*flops(T) "
                                     f"fitted and summed over the run's {wl['new_tokens']} steps",
                           "window_seconds": [round(v, 4) for v in secs]}
    return out


def parity_vs_cpu(device_ids, cpu_ids) -> dict:
    """Sequence 0's first device ids against the ids the CPU reference leg
    generated (same weights, prompt and RNG seed)."""
    dev = [int(t) for t in device_ids[:len(cpu_ids)]]
    ref = [int(t) for t in cpu_ids]
    first = next((i for i, (a, b) in enumerate(zip(dev, ref)) if a != b), None)
    return {"ids_compared": len(ref), "ids_equal": sum(a == b for a, b in zip(dev, ref)),
            "first_mismatch": first, "reference": "oracle port of the reference CPU loop (sequence 0)"}


def seqs_of(wl: dict, world: int, rank: int) -> tuple[int, int]:
    """(first sequence, count) of this rank."""
    if wl["seqs_total"]:
        return shard(wl["seqs_total"], world, rank)
    return rank * wl["seqs_per_gpu"], wl["seqs_per_gpu"]


def workload_config(wl: dict, world: int) -> dict:
    """The `config` object of a bench line (both arms print the same one)."""
    m = wl["model"]
    _, count = seqs_of(wl, world, 0)
    plen = wl["prompt_len"]
    wdt = wl.get("weight_dtype", "fp32")
    return {"workload": wl["name"], "model": model_name(m),
            "sequences_per_gpu": count, "prompt_len": plen if isinstance(plen, int) else list(plen),
            "new_tokens": wl["new_tokens"], "weights": wdt,
            "parallelism": f"request-parallel x{world} (independent sequences, no collective)",
            "l2": f"inputs larger than L2: every decode step streams {weight_bytes(m, wdt) / 1e6:.0f} MB "
                  f"of weights"}


def run_reference(args, wl):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(wl, full_run=(i == args.warmup + args.steps - 1))
        if i >= args.warmup:
            steps.append(r)
    toks = sum(len(r["ids"]) for r in steps)
    secs = sum(r["seconds"] for r in steps)
    v = toks / secs
    last = steps[-1]
    line = {"impl": "reference", "metric": "decode tokens/s", "value": v, "unit": "tokens/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / len(steps),
            "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random weights and prompt ids)",
            "config": workload_config(wl, world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": last["cores"], "cpu_model": last["cpu_model"],
                             "kind": "port", "sample": last["sample"], "full_run": last.get("full_run")},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def build_fingerprint(lib_path: str):
    """The source fingerprint the library file was built from (written beside
    it by the build), or None."""
    try:
        with open(lib_path + ".flags") as f:
            return json.load(f).get("sources_sha256")
    except (OSError, ValueError):
        return None


def recorded_traffic(workload: str, lib_path: str):
    """DRAM bytes per decode step from the traffic record, if it was measured
    on a library built from the same sources and flags; else None."""
    try:
        with open(TRAFFIC_RECORD) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None
    r = rec.get(workload)
    fp = build_fingerprint(lib_path)
    if not r or fp is None or r.get("build_sha256") != fp:
        return None
    return float(r["dram_bytes_per_step"])


def record_traffic(csv_path: str, workload: str, kernel: str, steps_per_launch: int) -> None:
    """Writes the traffic record from an ncu --csv capture of one or more
    launches of `kernel` with dram__bytes_read.sum and dram__bytes_write.sum
    (bytes, or the unit ncu prints), keyed by the build's source fingerprint."""
    import csv
    import __graft_entry__ as graft
    unit = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}
    per_launch: dict[str, float] = {}
    with open(csv_path) as f:
        lines = [ln for ln in f if ln.startswith('"')]
    for row in csv.DictReader(lines):
        if kernel not in row.get("Kernel Name", "") or not row.get("Metric Name", "").startswith("dram__bytes_"):
            continue
        v = float(row["Metric Value"].replace(",", "")) * unit.get(row.get("Metric Unit", "byte"), 1)
        per_launch[row["ID"]] = per_launch.get(row["ID"], 0.0) + v
    if not per_launch:
        raise SystemExit(f"no dram__bytes rows for {kernel} in {csv_path}")
    rec = {}
    if os.path.exists(TRAFFIC_RECORD):
        with open(TRAFFIC_RECORD) as f:
            rec = json.load(f)
    lib = graft.load_package().library_path()
    rec[workload] = {"kernel": kernel, "launches": len(per_launch), "steps_per_launch": steps_per_launch,
                     "dram_bytes_per_step": sum(per_launch.values()) / len(per_launch) / steps_per_launch,
                     "build_sha256": build_fingerprint(lib)}
    with open(TRAFFIC_RECORD, "w") as f:
        json.dump(rec, f, indent=1)
    print(json.dumps(rec[workload]))


def kernel_times(step, torch) -> None:
    """One step under the CUDA activity profiler: launches, total and mean
    device time per kernel (warm, in the step's own order and overlap, so
    the figures add up to the step; ncu's replayed times are cold and
    serialised), and the span from the first kernel's start to the last's end."""
    import collections
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    t0, t1 = None, None
    for ev in prof.events():
        if ev.device_type.name != "CUDA":
            continue
        agg[ev.name][0] += 1
        agg[ev.name][1] += ev.device_time_total
        t0 = ev.time_range.start if t0 is None else min(t0, ev.time_range.start)
        t1 = ev.time_range.end if t1 is None else max(t1, ev.time_range.end)
    total = sum(v[1] for v in agg.values())
    print(f"{sum(v[0] for v in agg.values())} kernels, {total / 1000:.2f} ms device time, "
          f"span {(t1 - t0) / 1000 if t0 is not None else 0:.2f} ms")
    print("| kernel | launches | total ms | share | mean us |")
    print("|---|---:|---:|---:|---:|")
    for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"| {name.split('(')[0].replace('void ', '')} | {n} | {t / 1000:.3f} | {100 * t / total:.1f} % | "
              f"{t / n:.2f} |")


def main():
    args = parse()
    if args.record_traffic:
        record_traffic(args.record_traffic, args.workload, args.record_kernel, args.record_steps_per_launch)
        return
    wl = dict(WORKLOADS[args.workload])
    default_wl = not args.new_tokens
    if args.new_tokens:
        wl["new_tokens"] = args.new_tokens
        wl["name"] += f" [new tokens overridden: {args.new_tokens}]"
    if args.impl == "reference":
        run_reference(args, wl)
        return
    import torch
    import torch.distributed as dist
    import __graft_entry__ as graft

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    pkg = graft.load_package()
    m = wl["model"]
    cfg = pkg.ModelConfig(**m)
    first, count = seqs_of(wl, world, rank)
    params = pkg.init_params(cfg, WEIGHT_SEED)
    wdt = wl.get("weight_dtype", "fp32")
    be = pkg.B200Backend(cfg, params, devices=[local], max_seqs=max(count, 1), weight_dtype=wdt)
    del params
    # a real (non-legacy) stream: its handle is what the library launches on,
    # and the CUDA events below are recorded on the same stream
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    be.set_stream(stream.cuda_stream)
    plen, new = wl["prompt_len"], wl["new_tokens"]
    prompts = prompts_for(first, count, plen, m["vocab_size"])
    lens = [len(p) for p in prompts]
    seeds = [1 + first + i for i in range(count)]
    dev = torch.device("cuda", local)
    d_prompts = torch.from_numpy(np.concatenate(prompts)).to(dev)
    d_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    d_out = torch.zeros((count, new), dtype=torch.int32, device=dev)
    d_cnt = torch.zeros((count,), dtype=torch.int32, device=dev)
    gen_kw = dict(max_new_tokens=new, temperature=wl["temperature"], top_k=wl["top_k"],
                  repetition_penalty=wl["penalty"], no_repeat_ngram_size=wl["ngram"])

    def step_device():
        be.generate_device(d_prompts.data_ptr(), d_lens.data_ptr(), lens, out_tokens_ptr=d_out.data_ptr(),
                           out_counts_ptr=d_cnt.data_ptr(), seeds=seeds, **gen_kw)

    def step_host():
        return be.generate_batch([p.tolist() for p in prompts], new, wl["temperature"], wl["top_k"], seeds=seeds,
                                 repetition_penalty=wl["penalty"], no_repeat_ngram_size=wl["ngram"])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: inputs resident in HBM --------------------------------------
    for _ in range(args.warmup):
        step_device()
    barrier()
    if args.kernel_times:
        if world > 1:
            raise SystemExit("--kernel-times runs on one GPU")
        kernel_times(step_device, torch)
        return
    be.reset_stats()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step_device()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1)
    st = be.stats()
    ms_max = max_over_ranks(ms)
    counts = d_cnt.cpu().numpy()
    tokens_rank = int(counts.sum()) * args.steps
    tokens_total = tokens_rank * world if wl["seqs_total"] is None else None
    if tokens_total is None:
        t = torch.tensor([tokens_rank], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t)
        tokens_total = int(t.item())
    value = tokens_total / (ms_max / 1000.0)

    # ---- per-step decode time (the roofline's unit): long minus short run ---
    def timed(fn, reps=2):
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        barrier()
        return a.elapsed_time(b) / reps

    short_kw = dict(gen_kw, max_new_tokens=1)
    be.reset_stats()
    t_long = timed(step_device)
    persistent = be.stats()["persistent_steps"] > 0
    t_short = timed(lambda: be.generate_device(d_prompts.data_ptr(), d_lens.data_ptr(), lens,
                                               out_tokens_ptr=d_out.data_ptr(), out_counts_ptr=d_cnt.data_ptr(),
                                               seeds=seeds, **short_kw))
    step_ms = (t_long - t_short) / max(new - 1, 1)
    bytes_step = weight_bytes(m, wdt) + float(np.mean(
        [sum(sequence_bytes(m, min(L0 + n, m["context_length"])) for L0 in lens) for n in range(1, new)]))
    achieved_gbs = bytes_step / (step_ms / 1000.0) / 1e9
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    if wl.get("bound") == "tensor":
        # every step re-forwards each sequence's full window
        flops_step = count * flops_per_sequence_step(m, m["context_length"])
        roofline = {"bound": "tensor", "kernel": "k_gemm_tc (tcgen05 3xTF32 GEMM) + k_attn_prefill_tc",
                    "achieved": flops_step / (step_ms / 1000.0) / 1e12,
                    "peak": float(peaks.get("bf16_tflops", 1590.0)), "unit": "TFLOP/s",
                    "peak_source": ("measured (MEASURED_PEAKS.json bf16_tflops; the GEMMs run TF32 with 3 MMAs per "
                                    "product for fp32 parity, and the TF32 dense rate is half the bf16 rate)")
                    if peaks else "fallback", "traffic": None, "step_ms": step_ms,
                    "algorithmic_flops_per_step": flops_step}
        roofline["frac"] = roofline["achieved"] / roofline["peak"]
    else:
        peak = float(peaks.get("hbm_gbs", 6650.0))
        roofline = {"bound": "hbm",
                    "kernel": "k_decode_mega (persistent decode kernel: cp.async.bulk weight stream, on-device "
                              "sampler)" if persistent else "decode step (CUDA graph replay of the step kernels)",
                    "achieved": achieved_gbs, "peak": peak, "unit": "GB/s", "frac": achieved_gbs / peak,
                    "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback",
                    "traffic": recorded_traffic(args.workload, pkg.library_path()) if default_wl else None,
                    "traffic_unit": "bytes per decode step: ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                    "workload's launch / its steps, recorded for this build (same source fingerprint; else null)",
                    "step_ms": step_ms, "algorithmic_bytes_per_step": bytes_step}

    # ---- e2e: the public host-buffer call, copies inside the timed region ----
    if args.skip_e2e:
        step_host = step_device
    step_host()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        res = step_host()
    b.record(stream)
    barrier()
    if args.skip_e2e:
        res = [d_out[i, :int(c)].cpu().numpy() for i, c in enumerate(d_cnt.cpu().numpy())]
    e2e_ms = max_over_ranks(a.elapsed_time(b))
    e2e_tokens = sum(len(r) for r in res) * args.steps * (world if wl["seqs_total"] is None else 1)
    if wl["seqs_total"] is not None and world > 1:
        t = torch.tensor([float(sum(len(r) for r in res) * args.steps)], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        e2e_tokens = int(t.item())
    e2e = {"value": e2e_tokens / (e2e_ms / 1000.0), "unit": "tokens/s",
           "h2d_bytes_per_step": int(sum(lens) * 4 + count * 4), "d2h_bytes_per_step": int(count * new * 4 + count * 4)}

    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference_sample(wl)
            cpu.pop("seconds", None)
            parity = parity_vs_cpu(res[0], cpu.pop("ids"))
        except Exception as ex:  # the baseline is informational; never fail the bench on it
            cpu = {"error": str(ex)}

    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, uniform-random prompt ids)",
            "config": workload_config(wl, world),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": e2e,
            "gpu_launches": int(st.get("kernel_launches", 0)),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
