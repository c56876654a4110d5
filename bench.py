#!/usr/bin/env python
"""Benchmark: Q4_0 decode tok/s of the Qwen2.5-0.5B architecture on B200, through libmatvec_b200.

Workload (config 3 of the reference's benchmark): a seeded synthetic Qwen2.5-0.5B-shaped .qwb (Q4 layer
matrices, Q8 65,536-row head, 390 MiB), a 128-token seeded prompt fed position by position (untimed), then
greedy decode. One step = 128 greedy tokens from the filled prompt cache (positions 127..254).

  value      device time (CUDA events on the model's stream) of K steps, each an asynchronous rewind to
             position 127 plus 128 launches of the captured decode-step graph; tok/s over all ranks.
  e2e        the same metric through the public C ABI with host buffers: per step mvb_qwen_rewind (state copied
             from pinned host memory) and mvb_qwen_decode (128 ids copied back to host memory), host wall clock.
  roofline   the dominant matvec kernel kind of the step (the path's kernel; every kind, attention included, is
             listed in per_kind with its share). Times come from the step exactly as the graph runs it (programmatic
             dependent launch included), every kernel stamping the GPU's global timer (mvb_qwen_stamps): a kernel's
             time is its last CTA's end minus the previous kernel's, so the kinds partition the step. Median of 5
             steps at the middle decode position (position 191), against MEASURED_PEAKS.json's HBM bandwidth.
             `traffic` is the DRAM bytes per launch of an ncu capture (profiles/traffic_per_launch.txt), given only
             when that capture was taken on the kernel sources of this tree (their hash is stamped in the file).
  cpu_baseline  the reference's own CPU build (oracle/_ref/qwen, -O3 -fopenmp -ffp-contract=off) on the same
             file and prompt, all host cores, its own "generated tok/s": median of K runs (the same count as the
             reference arm's steps).
  dropin     the reference's unchanged qwen.c linked against this library (oracle/_ref/qwen_b200: 200 synchronous
             fpga_matvec4 calls per token through the drop-in C ABI), same file and prompt, its own "generated tok/s",
             plus the library's per-call breakdown of fpga_matvec4 (MATVEC_STATS=1 run).
  sharded    config 5 (row-sharded 131072x8192 Q4 and the 151936-row Q8 head, batch 1 and 32) over all N ranks with
             the all-gather fused into the kernel (mvb_gather_*), beside the plain matvec + NCCL all-gather, each
             gathered vector checked bit for bit against the unsharded matvec (or matmul) of the whole matrix.
  runq, sweep, prefill_gemm   (rank 0 at N = 1) configs 1 and 2 (runq.c's stories15M / stories110M models decoded
             on the device, runq.c's CPU build beside them) and config 4 (the isolated matvec at M = 1 and the
             tensor-core matmul at M = 16 / 128 / 512, with bit-identity against per-token matvecs).
Every decode step reads the 263.7 MB of weights of a token, more than the 126 MB L2, so no flush is needed.

--impl reference times the reference's CPU implementation (oracle/_ref/qwen) on the same workload: K runs after
W warm-up runs, each one qwen.c generation of 128 greedy tokens from the 128-token prompt.
Multi-GPU (torchrun): the 0.5B decode does not shard; every rank runs an independent replica (weak scaling), and
the sharded block measures the one collective of the design.
"""
import argparse
import importlib.util
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "local-llama-pynq-z2_b200")
REF_QWEN = os.path.join(ROOT, "oracle", "_ref", "qwen")
REF_QWEN_B200 = os.path.join(ROOT, "oracle", "_ref", "qwen_b200")
DATA = os.environ.get("MVB_DATA", "/tmp/mvb_data")
METRIC = "Q4_0 decode tok/s (Qwen2.5-0.5B arch, 1 B200); matvec HBM GB/s vs peak"
PROMPT_LEN, GEN = 128, 128
PUBLISHED_TOKS = 3.7  # reference README: Qwen2.5-Coder-0.5B Q4_0 decode, FPGA matvec, 2 threads (PYNQ-Z2)
WORKLOAD = ("qwen2.5-0.5b-arch Q4_0 decode (config 3): synthetic seeded .qwb (Q4 layers, Q8 65536-row head), "
            "128-token prompt then 128 greedy tokens per step")
MATVEC_KINDS = ("qkv", "o_proj", "gate_up", "down", "head")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")


# the sources the decode step's kernels are compiled from (qwen_decode.cu and what it includes)
DECODE_SOURCES = ("qwen_decode.cu", "decode_kernels.cuh", "matvec_kernels.cuh", "prefill_kernels.cuh", "expf_ref.h",
                  "mvb_runtime.h")


def kernel_sources_sha():
    """Short hash of the decode step's kernel sources: names the code an ncu capture of the step covers."""
    import hashlib
    h = hashlib.sha256()
    for f in DECODE_SOURCES:
        h.update(f.encode())
        h.update(open(os.path.join(PKG, "csrc", f), "rb").read())
    return h.hexdigest()[:12]


def decode_config(world):
    """The `config` object of both arms' decode lines (the same workload and keys)."""
    return {"workload": WORKLOAD, "prompt_tokens": PROMPT_LEN, "gen_tokens_per_step": GEN, "replicas": world,
            "l2": "no flush: each token reads 263.7 MB of weights > 126 MB L2",
            "baseline": "3.7 tok/s, reference README.md:36 (PYNQ-Z2 FPGA)"}


def load_pkg():
    spec = importlib.util.spec_from_file_location("mvb", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mvb"] = mod
    spec.loader.exec_module(mod)
    return mod


def prompt_ids():
    import numpy as np
    return [int(t) for t in np.random.default_rng(3).integers(0, 151936, PROMPT_LEN)]


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples (200 ms) while running; summary() gives median SM MHz under load and active reasons."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p:
            self.p.terminate()
            self.p.wait()
        self.f.flush()
        rows = [r.split(", ") for r in open(self.f.name).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [v for v in sm if mx and v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def run_reference_qwen(model, prompt, n_gen, threads, binary=REF_QWEN, env_extra=None):
    """One qwen.c run (`binary`: the CPU build, or qwen_b200, the same source linked against this library) with
    --ids and greedy sampling: (its generated tok/s, tokens, prompt seconds, ids, stderr)."""
    env = dict(os.environ, OMP_NUM_THREADS=str(threads), **(env_extra or {}))
    r = subprocess.run([binary, model, "--ids", ",".join(map(str, prompt)), "-t", "0", "-n", str(n_gen), "-c", "512"],
                       capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        raise RuntimeError(os.path.basename(binary) + " failed: " + r.stderr[-500:])
    m = re.search(r"generated: (\d+) tokens, ([\d.]+) tok/s", r.stderr)
    pm = re.search(r"prompt: (\d+) tokens in ([\d.]+) s", r.stderr)
    ids = [int(t) for t in r.stdout.strip().split(",") if t]
    return float(m.group(2)), int(m.group(1)), float(pm.group(2)), ids, r.stderr


def reference_runs(path, prompt, runs, warmup, threads):
    """qwen.c's CPU build, `warmup` untimed runs then `runs` runs: (median generated tok/s, runs, last ids, last
    prompt seconds). The reference arm and the decode line's cpu_baseline both use this, with the same count."""
    for _ in range(warmup):
        run_reference_qwen(path, prompt, GEN, threads)
    res = [run_reference_qwen(path, prompt, GEN, threads) for _ in range(runs)]
    return statistics.median(r[0] for r in res), len(res), res[-1][3], res[-1][2]


def reference_sample(threads, runs):
    return (f"qwen.c CPU build (-O3 -fopenmp -ffp-contract=off, OMP_NUM_THREADS={threads}) on the same .qwb and "
            f"128-token prompt, {runs} runs of 128 greedy tokens; value = median of its own 'generated tok/s' (prompt "
            f"time excluded, as in the reference's report)")


def model_path(rank, world):
    sys.path.insert(0, PKG)
    import qwb
    if rank == 0:
        path = qwb.cached_qwb(DATA, qwb.QWEN05B, seed=0)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if rank != 0:
        path = qwb.cached_qwb(DATA, qwb.QWEN05B, seed=0)
    return path


def reference_arm(args, rank, world):
    if rank != 0:
        return
    if not os.path.exists(REF_QWEN):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/qwen was not built (the reference tree "
                                                              "was absent when __graft_entry__.build() ran)"}))
        return
    path = model_path(0, 1)
    threads = os.cpu_count()
    prompt = prompt_ids()
    value, runs, _, _ = reference_runs(path, prompt, args.steps, max(1, args.warmup), threads)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
            "steps": runs, "warmup": max(1, args.warmup), "ms_per_step": round(1000.0 * GEN / value, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / PUBLISHED_TOKS, 3),
            "dtype": "int4/int8->int32, fp32", "data": "synthetic", "config": decode_config(world),
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": reference_sample(threads, runs)},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def read_traffic(kind):
    """DRAM bytes (read + write) per launch of decode kernel `kind` from the committed ncu summary, with where it
    came from; None when the file's capture was taken on kernel sources other than this tree's."""
    sha_now = kernel_sources_sha()
    if not os.path.exists(TRAFFIC_FILE):
        return None, "no capture"
    sha_file, value = None, None
    for line in open(TRAFFIC_FILE):
        parts = line.split()
        if len(parts) == 2 and parts[0] == "sources":
            sha_file = parts[1]
        elif len(parts) == 2 and parts[0] == kind:
            value = float(parts[1])
    src = f"profiles/traffic_per_launch.txt (ncu capture of kernel sources {sha_file}; this tree {sha_now})"
    if sha_file != sha_now:
        return None, src + ": not this tree's kernels, so not used"
    return value, src


def step_roofline(dec, token, pos, reps=5, traffic=True):
    """Where the decode step's time goes, kernel kind by kernel kind, as the captured graph runs it: `reps` steps at
    (token, pos) with every kernel stamping the global timer (mvb_qwen_stamps). A kernel's time is its last CTA's
    end minus the previous kernel's (so the kinds partition the step, the kernel boundaries included); its
    in-kernel time starts when its first CTA got past the wait for the previous kernel. The roofline is the
    algorithmic GB/s of the dominant matvec kind (the path's kernel, decode_matvec_kernel) and of all matvecs
    together, against the measured HBM peak. The isolated per-kernel times (CUDA events around every kernel, no
    overlap, mvb_qwen_profile) are given beside them."""
    import numpy as np
    info = dec.kernel_info(pos)
    seg_runs, inside_runs, iso_runs = [], [], []
    for _ in range(reps):
        dec.rewind(token, pos, -1)
        st = dec.stamps()
        ends = st[:, 1]
        seg_runs.append(np.diff(np.concatenate([[0.0], ends])))
        inside_runs.append(st[:, 1] - st[:, 0])
        dec.rewind(token, pos, -1)
        iso_runs.append(dec.profile() * 1000.0)
    seg = np.median(seg_runs, axis=0)
    inside = np.median(inside_runs, axis=0)
    iso = np.median(iso_runs, axis=0)
    kinds = {}
    for (kind, layer, b), t, ti, tiso in zip(info, seg, inside, iso):
        k = kinds.setdefault(kind, {"launches": 0, "us": 0.0, "inside": 0.0, "iso": 0.0, "bytes": 0.0})
        k["launches"] += 1
        k["us"] += float(t)
        k["inside"] += float(ti)
        k["iso"] += float(tiso)
        k["bytes"] += b
    step_us = float(seg.sum())
    dom = max((k for k in kinds if k in MATVEC_KINDS), key=lambda k: kinds[k]["us"])
    peak, peak_kind = peaks()
    d = kinds[dom]
    achieved = d["bytes"] / (d["us"] * 1e-6) / 1e9
    mv_bytes = sum(kinds[k]["bytes"] for k in MATVEC_KINDS if k in kinds)
    mv_us = sum(kinds[k]["us"] for k in MATVEC_KINDS if k in kinds)
    all_bytes = sum(k["bytes"] for k in kinds.values())
    # the committed capture is of the Qwen decode's kernels; other models' steps run other instantiations
    traffic, traffic_src = read_traffic(dom) if traffic else (None, "no capture of this model's kernels")
    return {"bound": "hbm", "kernel": f"decode_matvec_kernel ({dom})", "kind": dom, "achieved": round(achieved, 1),
            "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
            "traffic": traffic, "traffic_source": traffic_src, "bytes_per_launch": round(d["bytes"] / d["launches"]),
            "us_per_launch": round(d["us"] / d["launches"], 3), "step_share": round(d["us"] / step_us, 4),
            "timing": "in the step graph with programmatic launch (mvb_qwen_stamps, %globaltimer): a kernel's time = "
                      "its last CTA's end minus the previous kernel's; median of 5 steps at position " + str(pos),
            "stamped_step_us": round(step_us, 2),
            "all_matvecs": {"bytes_per_token": round(mv_bytes), "us_per_token": round(mv_us, 2),
                            "achieved": round(mv_bytes / (mv_us * 1e-6) / 1e9, 1),
                            "frac": round(mv_bytes / (mv_us * 1e-6) / 1e9 / peak, 4)},
            "whole_step": {"bytes_per_token": round(all_bytes), "achieved": round(all_bytes / (step_us * 1e-6) / 1e9, 1),
                           "frac": round(all_bytes / (step_us * 1e-6) / 1e9 / peak, 4)},
            "isolated_step_us": round(float(iso.sum()), 2),
            "per_kind": {k: {"launches": v["launches"], "us_per_launch": round(v["us"] / v["launches"], 3),
                             "in_kernel_us": round(v["inside"] / v["launches"], 3),
                             "isolated_us": round(v["iso"] / v["launches"], 3),
                             "GBps": round(v["bytes"] / (v["us"] * 1e-6) / 1e9, 1),
                             "step_share": round(v["us"] / step_us, 4)} for k, v in kinds.items()}}


def our_arm(args, rank, world, local_rank):
    import numpy as np
    import torch
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
    mvb = load_pkg()
    path = model_path(rank, world)
    dec = mvb.QwenDecoder(path, ctx=512)
    cfg = dec.cfg
    stream = torch.cuda.ExternalStream(dec.stream_handle)
    prompt = prompt_ids()
    dec.prefill(prompt)
    pos0, tok0 = PROMPT_LEN - 1, prompt[-1]

    def device_steps(k):
        for _ in range(k):
            dec.rewind(tok0, pos0, PROMPT_LEN)
            dec.launch(GEN)

    def sync_all():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up
    device_steps(args.warmup)
    sync_all()
    # value: device-timed decode
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = getattr(torch.cuda.get_device_properties(local_rank), "uuid", None)
    clocks = Clocks(f"GPU-{uuid}" if uuid is not None else local_rank)
    sync_all()
    e0.record(stream)
    device_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1000.0)
    value = world * args.steps * GEN / t_dev
    # e2e: public C ABI with host buffers, host wall clock
    ids_first = None
    sync_all()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dec.rewind(tok0, pos0, PROMPT_LEN)
        ids = dec.decode(GEN)
        if ids_first is None:
            ids_first = ids.copy()
        elif not np.array_equal(ids, ids_first):
            raise RuntimeError("decode steps disagree")
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    e2e = world * args.steps * GEN / t_e2e
    # roofline: one instrumented step at the middle decode position, 5 repeats
    mid = pos0 + GEN // 2
    roofline = step_roofline(dec, tok0 if mid == pos0 else int(ids_first[mid - pos0 - 1]), mid)
    # prompt prefill through the public API (host wall clock, the call returns when the cache is written): the
    # batched path (tensor-core matmuls) and one decode step per fed token
    def timed_prefill(fn, reps=3):
        fn(prompt)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn(prompt)
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)
    t_pf = timed_prefill(dec.prefill)
    t_pf_tok = timed_prefill(dec.prefill_tokenwise)
    prefill = {"fed_tokens": PROMPT_LEN - 1, "ms": round(t_pf * 1000, 3),
               "tok_s": round((PROMPT_LEN - 1) / t_pf, 1), "tokenwise_ms": round(t_pf_tok * 1000, 3),
               "tokenwise_tok_s": round((PROMPT_LEN - 1) / t_pf_tok, 1),
               "how": "mvb_qwen_prefill (batched: tensor-core matmuls) and mvb_qwen_prefill_tokenwise (one decode "
                      "step per token); host wall clock of the synchronous call, median of 3"}
    dec.close()
    cpu, dropin = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and os.path.exists(REF_QWEN):
        threads = os.cpu_count()
        tps, runs, ref_ids, ref_prompt_s = reference_runs(path, prompt, args.steps, 1, threads)
        cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
               "sample": reference_sample(threads, runs), "same_ids_as_b200": ref_ids == ids_first.tolist()}
        prefill["reference_prompt_s"] = ref_prompt_s
    if rank == 0 and world == 1 and not args.no_cpu_baseline and os.path.exists(REF_QWEN_B200):
        dropin = dropin_block(path, prompt, ids_first.tolist(), local_rank)
    extra = {}
    if rank == 0 and world == 1 and not args.no_extra:
        extra = extra_blocks(args, mvb)
    sharded = None
    if not args.no_sharded:
        sharded = sharded_cases(rank, world, max(args.steps, 50), max(args.warmup, 3), dist)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(1000.0 * t_dev / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": round(value / PUBLISHED_TOKS, 2),
                "dtype": "int4/int8->int32, fp32", "data": "synthetic", "config": decode_config(world),
                "roofline": roofline, "cpu_baseline": cpu,
                "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 32,
                        "d2h_bytes_per_step": 4 * GEN + 32},
                "gpu_launches": args.steps * GEN * cfg["kernels_per_step"], "clocks": clk, "prefill": prefill,
                "dropin": dropin, "sharded": sharded, **extra}
        print(json.dumps(line), flush=True)


CONFIG4_MATVEC_SHAPES = [(896, 896, 4), (896, 128, 4), (896, 4864, 4), (4864, 896, 4), (896, 65536, 8)]


def extra_blocks(args, mvb):
    """The other configs of the reference's benchmark, measured on one GPU beside the decode line (rank 0, N = 1):
    configs 1 and 2 (runq.c's stories15M / stories110M models decoded on the device, with runq.c's CPU build timed
    beside them) and config 4 (the isolated matvec at M = 1 and the tensor-core matmul at M = 16 / 128 / 512)."""
    import argparse as ap
    import torch
    ns = ap.Namespace(model="", gs=32, steps=max(1, min(args.steps, 10)), warmup=max(1, min(args.warmup, 3)),
                      no_cpu_baseline=args.no_cpu_baseline)
    keep = ("metric", "value", "unit", "us_per_token", "steps", "flushed", "e2e", "cpu_baseline", "kernels_per_token")
    runq = []
    for l in runq_results(ns):
        r = {k: l[k] for k in keep}
        r["workload"] = l["config"]["workload"]
        r["stamped_step_us"] = l["roofline"]["stamped_step_us"]
        runq.append(r)
    peak, peak_kind = peaks()
    sweep = sweep_results(mvb, torch, CONFIG4_MATVEC_SHAPES, [])
    gemm, int8_peak = prefill_results(mvb, torch, PREFILL_SHAPES, (16, 128, 512), time_matvecs=False)
    return {"runq": {"how": "configs 1 and 2 (bench.py --mode runq, fewer steps); value = device tok/s with the "
                            "weights warm in L2, flushed = each token after a 256 MB L2 flush", "results": runq},
            "sweep": {"how": "config 4 at M = 1: one matvec per call in a CUDA graph, weights rotated past L2; "
                             "GB/s of the algorithmic bytes", "peak": peak, "peak_source": f"{peak_kind} hbm_gbs",
                      "results": sweep},
            "prefill_gemm": {"how": "config 4 at M = 16 / 128 / 512: the tcgen05 int8 matmul (mvb_gemm4) per call in "
                                    "a CUDA graph, weights rotated past L2; same = equal bit for bit to one matvec "
                                    "per token (M <= 128)", "int8_peak_TOPS": int8_peak, "results": gemm}}


def dropin_block(path, prompt, ids_b200, gpu):
    """The drop-in boundary as the reference's users would run it: qwen.c unchanged, compiled with -DFPGA against
    include/matvec_fpga.h and linked to this library (oracle/_ref/qwen_b200), on the same file and prompt: each
    matvec is one synchronous fpga_matvec4 call (200 per token) with host buffers. Median of 3 runs of its own
    'generated tok/s'; then one run with MATVEC_STATS=1, whose fpga_close() reports the per-call breakdown."""
    threads = os.cpu_count()
    env = {"FPGA_MEMIDX": str(gpu)}
    runs = [run_reference_qwen(path, prompt, GEN, threads, REF_QWEN_B200, env) for _ in range(3)]
    _, _, _, _, err = run_reference_qwen(path, prompt, GEN, threads, REF_QWEN_B200, dict(env, MATVEC_STATS="1"))
    stats = None
    m = re.search(r"matvec stats: (\{.*\})", err)
    if m:
        stats = json.loads(m.group(1))
    return {"value": round(statistics.median(r[0] for r in runs), 2), "unit": "tok/s", "runs": len(runs),
            "how": "qwen.c unchanged, -DFPGA, linked to libmatvec_b200.so (oracle/_ref/qwen_b200); its own "
                   "'generated tok/s' (prompt excluded); 200 synchronous fpga_matvec4 calls per token",
            "same_ids_as_b200": runs[-1][3] == ids_b200, "per_call": stats}


# ---- isolated-kernel modes (not the driver's default line) ----

def _alg_bytes(n, d, bits, scale_bytes=2, gs=32):
    """Algorithmic bytes of one matvec call: weights, scales, int8 activations + scales, fp32 outputs."""
    return d * n * bits // 8 + d * (n // gs) * scale_bytes + n + (n // gs) * 4 + 4 * d


def _rand_matrix(torch, n, d, bits, copies, gen):
    w = [torch.randint(0, 256, (d * n * bits // 8,), dtype=torch.uint8, device="cuda", generator=gen)
         for _ in range(copies)]
    # fp16 scales in [1e-3, 2e-2] as bit patterns
    s = [(torch.rand(d * (n // 32), device="cuda", generator=gen) * 0.019 + 0.001).half().view(torch.int16)
         for _ in range(copies)]
    return w, s


def _time_graph(torch, fn, reps):
    """Per-call device time (s) of fn() captured reps times in one CUDA graph (host launch cost excluded)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(5):
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1000.0 / reps)
    del g
    return statistics.median(times)


def sweep_results(mvb, torch, shapes, runq_shapes, emit=False):
    """The isolated matvec per shape (graph of calls, weights rotated past L2): runq's int8 fp32-scale matvec for
    runq_shapes ((n, d), group size 32) and matvec4 for shapes ((n, d, bits), fp16 scales). Returns one dict per
    shape (us, GB/s of the algorithmic bytes, fraction of the measured HBM peak)."""
    gen = torch.Generator(device="cuda").manual_seed(0)
    peak, _ = peaks()
    out_lines = []
    for n, d in runq_shapes:
        gs = 32
        b = _alg_bytes(n, d, 8, scale_bytes=4, gs=gs)
        copies = max(2, min(4096, -(-300 * 2**20 // b)))
        w = [torch.randint(-127, 128, (d * n,), dtype=torch.int8, device="cuda", generator=gen) for _ in range(copies)]
        sc = [torch.rand(d * (n // gs), device="cuda", generator=gen) * 0.019 + 0.001 for _ in range(copies)]
        xq = torch.randint(-127, 128, (n,), dtype=torch.int8, device="cuda", generator=gen)
        xs = torch.rand(n // gs, device="cuda", generator=gen) * 0.05
        out = torch.empty(d, device="cuda")
        reps = max(copies, 64)
        t = _time_graph(torch, lambda i: mvb.matvec(w[i % copies], sc[i % copies], xq, xs, out, n, d, gs), reps)
        line = {"shape": f"{d}x{n} Q8 fp32-scale (runq)", "us": round(t * 1e6, 3), "GBps": round(b / t / 1e9, 1),
                "frac": round(b / t / 1e9 / peak, 4), "bytes": b, "copies": copies}
        out_lines.append(line)
        if emit:
            print(json.dumps(line), flush=True)
        del w, sc
        torch.cuda.empty_cache()
    for n, d, bits in shapes:
        b = _alg_bytes(n, d, bits)
        copies = max(2, min(4096, -(-300 * 2**20 // b)))
        w, sc = _rand_matrix(torch, n, d, bits, copies, gen)
        xq = torch.randint(-127, 128, (n,), dtype=torch.int8, device="cuda", generator=gen)
        xs = torch.rand(n // 32, device="cuda", generator=gen) * 0.05
        out = torch.empty(d, device="cuda")
        reps = max(copies, 64)
        t = _time_graph(torch, lambda i: mvb.matvec4(w[i % copies], sc[i % copies], xq, xs, out, n, d, bits), reps)
        line = {"shape": f"{d}x{n} Q{bits}", "us": round(t * 1e6, 3), "GBps": round(b / t / 1e9, 1),
                "frac": round(b / t / 1e9 / peak, 4), "bytes": b, "copies": copies,
                "rows_per_tile": mvb.rows_per_tile(n, d)}
        out_lines.append(line)
        if emit:
            print(json.dumps(line), flush=True)
        del w, sc
        torch.cuda.empty_cache()
    return out_lines


def sweep_mode(args):
    """Config 4: the isolated matvec at the Qwen2.5-0.5B layer shapes and the heads, plus the large sharded
    matrix on one GPU; inputs rotate through copies larger than 2x L2 so every call reads HBM."""
    import torch
    mvb = load_pkg()
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    shapes, runq_shapes = SWEEP_SHAPES, SWEEP_RUNQ_SHAPES
    if args.only:
        shapes = [sh for sh in shapes if f"{sh[1]}x{sh[0]}" == args.only]
        runq_shapes = [sh for sh in runq_shapes if f"{sh[1]}x{sh[0]}" == args.only]
    out_lines = sweep_results(mvb, torch, shapes, runq_shapes, emit=True)
    print(json.dumps({"mode": "sweep", "peak": peak, "peak_source": f"{peak_kind} hbm_gbs", "results": out_lines}))


SWEEP_SHAPES = [(896, 896, 4), (896, 128, 4), (896, 4864, 4), (4864, 896, 4), (896, 1152, 4), (896, 65536, 8),
                (896, 151936, 8), (8192, 131072, 4)]  # (n columns, d rows, weight bits): fp16-scale matvecs
SWEEP_RUNQ_SHAPES = [(288, 288), (288, 768), (768, 288), (288, 32000), (768, 768), (768, 2048), (2048, 768),
                     (768, 32000)]  # runq's int8 weights with fp32 scales at the stories15M / stories110M shapes


def reference_sweep(args):
    """Config 4 on the host cores: the reference's own CPU matvec, timed per sweep shape. qwen.c's matmul_cpu
    (qwen.c:436-456, OpenMP over rows) for the Q4/Q8 fp16-scale shapes and runq.c's matmul (runq.c:430-458) for the
    fp32-scale shapes, both compiled unchanged into oracle/_ref/ with -O3 -fopenmp -ffp-contract=off, with every
    host core. Weights rotate through copies that together exceed 512 MB (beyond any host's last-level cache), so
    every call streams its matrix from DRAM, as the device sweep streams it from HBM. Each shape runs calls for
    about a second (bounded sample) after one warm-up pass over all copies; GB/s uses the same algorithmic bytes."""
    import ctypes as C
    import numpy as np
    threads = os.cpu_count()
    os.environ["OMP_NUM_THREADS"] = str(threads)  # read by libgomp when the harness library loads below
    libs = {name: os.path.join(ROOT, "oracle", "_ref", name) for name in ("libref_qwen.so", "libref_runq.so")}
    if not all(os.path.exists(p) for p in libs.values()):
        print(json.dumps({"mode": "sweep", "impl": "reference",
                          "unavailable": "oracle/_ref was not built (the reference tree was absent at build time)"}))
        return
    lq, lr = C.CDLL(libs["libref_qwen.so"]), C.CDLL(libs["libref_runq.so"])
    vp, sz = C.c_void_p, C.c_size_t
    lq.ref_qwen_time_matmul_cpu.restype = lr.ref_runq_time_matmul_cpu.restype = C.c_double
    lq.ref_qwen_time_matmul_cpu.argtypes = lr.ref_runq_time_matmul_cpu.argtypes = [
        vp, vp, vp, sz, sz, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int]
    rng = np.random.default_rng(0)
    pool = 512 * 2**20
    shapes = [(n, d, 8, "runq") for n, d in SWEEP_RUNQ_SHAPES] + [(n, d, b, "qwen") for n, d, b in SWEEP_SHAPES]
    if args.only:
        shapes = [sh for sh in shapes if f"{sh[1]}x{sh[0]}" == args.only]
    wbytes_max = max(d * n * b // 8 for n, d, b, _ in shapes) if shapes else 0
    wpool = np.frombuffer(rng.bytes(max(pool, wbytes_max)), np.uint8)  # weight bytes: uniform int4 nibbles / int8
    # fp16 scale patterns in [1e-3, 2e-2]; fp32 scales the same range; at most 1/8 of a weight byte per weight byte
    s16 = (rng.random(wpool.size // 8 // 2 + 1) * 0.019 + 0.001).astype(np.float16).view(np.uint16)
    s32 = (rng.random(wpool.size // 8 // 4 + 1) * 0.019 + 0.001).astype(np.float32)
    results = []
    for n, d, bits, kind in shapes:
        wbytes, ng = d * n * bits // 8, d * (n // 32)
        copies = max(1, min(wpool.size // wbytes, 4096))
        x = rng.standard_normal(n).astype(np.float32)
        amax = np.abs(x.reshape(-1, 32)).max(axis=1)
        xs = (amax / np.float32(127)).astype(np.float32)  # activations: N(0, 1) quantized per group of 32
        xq = np.clip(np.rint(x / np.repeat(xs, 32)), -127, 127).astype(np.int8)
        out = np.empty(d, np.float32)
        if kind == "qwen":
            fn, sc, scb = lq.ref_qwen_time_matmul_cpu, s16, 2
            b = _alg_bytes(n, d, bits)
            label = f"{d}x{n} Q{bits}"
        else:
            fn, sc, scb = lr.ref_runq_time_matmul_cpu, s32, 4
            b = _alg_bytes(n, d, 8, scale_bytes=4)
            label = f"{d}x{n} Q8 fp32-scale (runq)"
        call = lambda reps: fn(out.ctypes.data, wpool.ctypes.data, sc.ctypes.data, wbytes, ng, copies,
                               xq.ctypes.data, xs.ctypes.data, n, d, bits if kind == "qwen" else 32, reps)
        t1 = call(copies) / copies  # warm-up over every copy (first touch of the pool pages)
        reps = max(3, min(1_000_000, int(1.0 / max(t1, 1e-7))))
        t = call(reps) / reps
        line = {"impl": "reference", "shape": label, "us": round(t * 1e6, 3), "GBps": round(b / t / 1e9, 2),
                "bytes": b, "copies": copies, "calls": reps}
        results.append(line)
        print(json.dumps(line), flush=True)
    cpu = ""
    try:
        cpu = next((l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name")), "")
    except OSError:
        pass
    print(json.dumps({"mode": "sweep", "impl": "reference", "cores": threads, "cpu": cpu,
                      "sample": "the reference's matmul_cpu (qwen.c) / matmul (runq.c), -O3 -fopenmp "
                                "-ffp-contract=off, OMP_NUM_THREADS = all host cores, about 1 s of calls per shape, "
                                "weights rotated through >= 512 MB of copies", "results": results}))


def prefill_results(mvb, torch, shapes, ms, time_matvecs=True, emit=False):
    """The tensor-core matmul (mvb_gemm4) per shape ((n, d, bits)) and token count in ms (graph of calls, weights
    rotated past L2), with `same`: its output equals one matvec4 call per token, bit for bit (M <= 128), and, when
    time_matvecs, those M matvec calls timed too. Returns one dict per (shape, M)."""
    gen = torch.Generator(device="cuda").manual_seed(0)
    bf16 = 1590.0
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(mp):
        bf16 = float(json.load(open(mp)).get("bf16_tflops", bf16))
    int8_peak = 2 * bf16
    out_lines = []
    for n, d, bits in shapes:
        wb = d * n * bits // 8 + d * (n // 32) * 2
        copies = max(2, min(4096, -(-300 * 2**20 // wb)))
        w, sc = _rand_matrix(torch, n, d, bits, copies, gen)
        for m in ms:
            xq = torch.randint(-127, 128, (m, n), dtype=torch.int8, device="cuda", generator=gen)
            ldx = (m + 3) // 4 * 4
            xs = torch.rand((n // 32, ldx), device="cuda", generator=gen) * 0.05
            out = torch.empty((m, d), device="cuda")
            reps = max(min(copies, 256), 16)
            t = _time_graph(torch, lambda i: mvb.gemm4(w[i % copies], sc[i % copies], xq, xs, out, n, d, m, ldx, bits),
                            reps)
            status = mvb.gemm_status()
            # the same tokens, one matvec call each
            xs_tok = xs[:, :m].t().contiguous()
            out_mv = torch.empty((m, d), device="cuda")
            mv_reps = max(1, min(copies, 4096 // m))

            def per_token(i):
                for tk in range(m):
                    mvb.matvec4(w[i % copies], sc[i % copies], xq[tk], xs_tok[tk], out_mv[tk], n, d, bits)

            t_mv = _time_graph(torch, per_token, mv_reps) if m <= 128 and time_matvecs else None
            mvb.gemm4(w[0], sc[0], xq, xs, out, n, d, m, ldx, bits)
            per_token(0) if m <= 128 else None
            torch.cuda.synchronize()
            same = bool(torch.equal(out.view(torch.int32), out_mv.view(torch.int32))) if m <= 128 else None
            ops = 2.0 * m * d * n
            line = {"shape": f"{d}x{n} Q{bits}", "M": m, "us": round(t * 1e6, 2),
                    "TOPS": round(ops / t / 1e12, 1), "frac_int8": round(ops / t / 1e12 / int8_peak, 4),
                    "weight_GBps": round(wb / t / 1e9, 1), "group_results_per_s": round(m * d * (n // 32) / t / 1e12, 3),
                    "matvecs_us": round(t_mv * 1e6, 2) if t_mv else None,
                    "speedup_vs_matvecs": round(t_mv / t, 1) if t_mv else None, "same": same, "status": status}
            out_lines.append(line)
            if emit:
                print(json.dumps(line), flush=True)
        del w, sc
        torch.cuda.empty_cache()
    return out_lines, int8_peak


PREFILL_SHAPES = [(896, 896, 4), (896, 128, 4), (896, 4864, 4), (4864, 896, 4), (896, 65536, 8)]


def prefill_shapes(only):
    """The (columns, rows, bits) shapes of --mode prefill: config 4's, the one of them named by `only` (rows x
    columns), or any shape `only` names outside them (rows x columns, Q4 unless qN follows: 8192x8192, 65536x896q8);
    [] for a name that is neither."""
    if not only:
        return list(PREFILL_SHAPES)
    shapes = [sh for sh in PREFILL_SHAPES if f"{sh[1]}x{sh[0]}" == only]
    m = re.fullmatch(r"(\d+)x(\d+)(?:q([48]))?", only)
    if not shapes and m:
        shapes = [(int(m.group(2)), int(m.group(1)), int(m.group(3) or 4))]
    return shapes


def prefill_mode(args):
    """Config 4's batched part: the tensor-core prefill matmul (mvb_gemm4) with M = 16, 128 and 512 tokens on the
    Qwen2.5-0.5B layer shapes and the Q8 head, beside the same tokens as M calls of the matvec kernel (one per
    token, as the reference prefills). Weights rotate through copies larger than 2x L2. Reported per shape and M:
    us per call, int8 tensor ops 2*M*d*n per second against the int8 dense rate taken as twice the measured bf16
    peak (B200's int8 rate is twice its bf16 rate), weight GB/s, and the epilogue's rate of group results
    (M*d*n/32 per second); `same` says the GEMM's output equals the M matvecs' bit for bit."""
    import torch
    mvb = load_pkg()
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    shapes = prefill_shapes(args.only)
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    out_lines, int8_peak = prefill_results(mvb, torch, shapes, [args.m] if args.m else (16, 128, 512), emit=True)
    print(json.dumps({"mode": "prefill", "int8_peak_TOPS": int8_peak,
                      "peak_source": f"2 x {peak_kind} bf16_tflops" if os.path.exists(mp) else "2 x fallback bf16",
                      "results": out_lines}))


def prompt_mode(args):
    """Config 3's prompt phase alone: the batched prefill of the 127 fed prompt tokens (mvb_qwen_prefill:
    tensor-core matmuls, batched attention), K times after W warm-ups, device-timed with CUDA events on the
    model's stream around each call (the call synchronizes before returning)."""
    import torch
    mvb = load_pkg()
    torch.cuda.set_device(0)
    dec = mvb.QwenDecoder(model_path(0, 1), ctx=512)
    stream = torch.cuda.ExternalStream(dec.stream_handle)
    prompt = prompt_ids()
    for _ in range(args.warmup):
        dec.prefill(prompt)
    ts = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.prefill(prompt)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    dec.close()
    ms = statistics.median(ts)
    print(json.dumps({"mode": "prompt", "fed_tokens": PROMPT_LEN - 1, "ms": round(ms, 3),
                      "tok_s": round((PROMPT_LEN - 1) / ms * 1000, 1), "steps": args.steps, "warmup": args.warmup}))


def step_mode(args):
    """Config 3's decode alone, for profiling: load, batched prompt prefill, then K single decode steps (graph
    launches) after W warm-up steps, each device-timed on the model's stream; prints the median step time."""
    import torch
    mvb = load_pkg()
    torch.cuda.set_device(0)
    dec = mvb.QwenDecoder(model_path(0, 1), ctx=512)
    if args.full_head:
        dec.full_head(True)
    stream = torch.cuda.ExternalStream(dec.stream_handle)
    prompt = prompt_ids()
    dec.prefill(prompt)
    dec.launch(args.warmup)
    ts = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.launch(1)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    dec.close()
    ms = statistics.median(ts)
    print(json.dumps({"mode": "step", "head": "full vocabulary" if args.full_head else "trimmed (head_ids)",
                      "ms_per_token": round(ms, 4), "tok_s": round(1000 / ms, 1), "steps": args.steps,
                      "warmup": args.warmup}))


SHARDED_CASES = ((8192, 131072, 4), (896, 151936, 8))  # config 5: (n columns, d rows, weight bits)


def sharded_cases(rank, world, iters, warmup, dist):
    """Config 5 on `world` ranks (one per GPU; dist is torch.distributed, or None for one rank): each matrix
    row-sharded in contiguous blocks (rows per rank = ceil(d / world), the last block padded), every rank ending the
    step with the whole fp32 output. Timed per step with CUDA events, max over ranks: the fused kernel that stores its
    rows into every rank's output over NVLink (mvb_gather_matvec4 at batch 1, mvb_gather_gemm4 at batch 32: the
    reported number) and the plain matvec/matmul of the shard alone, each as `iters` calls captured in a CUDA graph
    (device time, no host launch cost between calls) and as calls launched one by one from Python (`*_eager_us`);
    and (world > 1) the plain call followed by an NCCL all-gather, with the all-gather alone, launched from Python.
    Every rank checks its gathered output bit for bit against the unsharded matvec (or matmul) of the whole matrix,
    and the NCCL path's result against the fused one."""
    import torch
    mvb = sys.modules.get("mvb") or load_pkg()
    peak, peak_kind = peaks()
    results = []

    def sync():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, graph=False):
        for i in range(warmup):
            fn(i)
        sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if graph:  # iters calls captured once, replayed: device time without host launch gaps
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                for i in range(iters):
                    fn(i)
            g.replay()
            sync()
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            del g
        else:
            e0.record()
            for i in range(iters):
                fn(i)
            e1.record()
            torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1000.0 / iters
        if dist:
            tt = torch.tensor([t], dtype=torch.float64, device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    def all_ranks(ok):
        if not dist:
            return bool(ok)
        t = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    def shard(q, rows, n, bits):
        """Rank q's block of copy 0 of the matrix (seeded by q): the same bytes on every rank."""
        g0 = torch.Generator(device="cuda").manual_seed(1000 + q)
        w, sc = _rand_matrix(torch, n, rows, bits, 1, g0)
        return w[0], sc[0]

    def connect(g):
        handles = [None] * world
        if dist:
            dist.all_gather_object(handles, g.handle())
        else:
            handles = [g.handle()]
        g.connect(handles)

    for n, d, bits in SHARDED_CASES:
        rows = -(-d // world)
        total = _alg_bytes(n, d, bits)
        b_local = _alg_bytes(n, rows, bits)
        copies = max(1, -(-300 * 2**20 // b_local))  # this rank's copies rotate past the 126 MB L2
        w0, s0 = shard(rank, rows, n, bits)
        w_more, s_more = _rand_matrix(torch, n, rows, bits, copies - 1,
                                      torch.Generator(device="cuda").manual_seed(1234 + rank)) if copies > 1 else ([], [])
        w, sc = [w0] + w_more, [s0] + s_more
        xq = torch.randint(-127, 128, (n,), dtype=torch.int8, device="cuda",
                           generator=torch.Generator(device="cuda").manual_seed(7))
        xs = torch.rand(n // 32, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9)) * 0.05
        m = 32
        xq32 = torch.randint(-127, 128, (m, n), dtype=torch.int8, device="cuda",
                             generator=torch.Generator(device="cuda").manual_seed(8))
        xs32 = torch.rand((n // 32, m), device="cuda", generator=torch.Generator(device="cuda").manual_seed(10)) * 0.05
        # the unsharded results of the whole (padded) matrix, from every rank's copy-0 block
        blocks = [shard(q, rows, n, bits) for q in range(world)]
        w_full = torch.cat([b[0] for b in blocks])
        s_full = torch.cat([b[1] for b in blocks])
        del blocks
        ref1 = torch.empty(rows * world, device="cuda")
        mvb.matvec4(w_full, s_full, xq, xs, ref1, n, rows * world, bits)
        ref32 = torch.empty((m, rows * world), device="cuda")
        mvb.gemm4(w_full, s_full, xq32, xs32, ref32, n, rows * world, m, m, bits)
        torch.cuda.synchronize()
        if mvb.gemm_status() != 0:
            raise RuntimeError("sharded: a matmul wait gave up")
        del w_full, s_full
        torch.cuda.empty_cache()
        for batch in (1, m):
            g = mvb.ShardGather(rank, world, rows, tokens=batch)
            connect(g)
            part = torch.empty((batch, rows), device="cuda")
            if batch == 1:
                fused = lambda i: g.matvec4(w[i % copies], sc[i % copies], xq, xs, n, bits)
                plain = lambda i: mvb.matvec4(w[i % copies], sc[i % copies], xq, xs, part, n, rows, bits)
            else:
                fused = lambda i: g.gemm4(w[i % copies], sc[i % copies], xq32, xs32, n, m, m, bits)
                plain = lambda i: mvb.gemm4(w[i % copies], sc[i % copies], xq32, xs32, part, n, rows, m, m, bits)
            t_fused = timed(fused, graph=True)
            t_plain = timed(plain, graph=True)
            t_fused_eager = timed(fused)
            t_plain_eager = timed(plain)
            sync()
            fused(0)
            torch.cuda.synchronize()
            got = g.output().clone()
            ref = ref1 if batch == 1 else ref32
            same = bool(torch.equal(got.view(torch.int32), ref.view(torch.int32))) and g.error() == 0
            line = {"shape": f"{d}x{n} Q{bits}", "batch": batch, "n_gpus": world, "rows_per_gpu": rows,
                    "us_per_step": round(t_fused * 1e6, 2), "GBps_total": round(total / t_fused / 1e9, 1),
                    "frac_of_aggregate_hbm": round(total / t_fused / 1e9 / (peak * world), 4),
                    "shard_alone_us": round(t_plain * 1e6, 2), "exchange_us": round((t_fused - t_plain) * 1e6, 2),
                    "fused_eager_us": round(t_fused_eager * 1e6, 2), "shard_alone_eager_us": round(t_plain_eager * 1e6, 2)}
            if batch > 1:
                line["tokens_per_s"] = round(batch / t_fused, 1)
            if dist and world > 1:
                full = torch.empty((world, batch, rows), device="cuda")
                ag = lambda i: dist.all_gather_into_tensor(full, part)
                nccl = lambda i: (plain(i), ag(i))
                line["nccl_path_us"] = round(timed(nccl) * 1e6, 2)
                line["nccl_allgather_us"] = round(timed(ag) * 1e6, 2)
                nccl(0)
                torch.cuda.synchronize()
                same = same and bool(torch.equal(full.permute(1, 0, 2).reshape(batch, world * rows).view(torch.int32),
                                                 got.view(batch, -1).view(torch.int32)))
            line["bit_identical"] = all_ranks(same)
            sync()  # no rank's kernel still stores into a buffer about to be freed
            g.close()
            sync()
            results.append(line)
        del w, sc
        torch.cuda.empty_cache()
    return {"collective": "fused peer stores over NVLink (mvb_gather_matvec4 at batch 1, mvb_gather_gemm4 at batch 32, "
                          "the reported us_per_step); NCCL all_gather_into_tensor after the plain call for comparison",
            "timing": "us_per_step and shard_alone_us: iters calls in one CUDA graph (device time); *_eager_us and the "
                      "NCCL figures: calls launched one by one from Python; max over ranks",
            "check": "every rank's gathered output equals the unsharded matvec/matmul of the whole matrix bit for bit "
                     "(and the NCCL path's)", "peak_per_gpu": peak, "peak_source": f"{peak_kind} hbm_gbs",
            "iters": iters, "results": results}


def sharded_mode(args, rank, world, local_rank):
    """Config 5 alone (the sharded block of the decode line): prints its results on rank 0."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    load_pkg()
    out = sharded_cases(rank, world, max(args.steps, 50), max(args.warmup, 3), dist if world > 1 else None)
    if rank == 0:
        print(json.dumps({"mode": "sharded", **out}), flush=True)


RUNQ_MODELS = {"stories15m": ("STORIES15M", "stories15M"), "stories110m": ("STORIES110M", "stories110M")}
RUNQ_PROMPT = 4


def run_reference_runq(path, prompt, npos, threads):
    """runq.c's CPU build (oracle/_ref/libref_runq.so: its own forward) on the same checkpoint and prompt in a child
    process with `threads` OpenMP threads: (tok/s over positions 1 .. npos-1, timed like runq.c:1024-1033 from the
    end of the first forward, greedy ids after the prompt)."""
    code = f"""
import sys, time
import numpy as np
sys.path.insert(0, {os.path.join(ROOT, 'oracle')!r})
import oracle
r = oracle.RefRunq()
r.open({path!r})
prompt, tok, ids = {list(prompt)!r}, {int(prompt[0])}, []
for pos in range({npos}):
    lg = r.forward(tok, pos)
    if pos == 0:
        t0 = time.perf_counter()
    tok = prompt[pos + 1] if pos + 1 < len(prompt) else int(r.lib.ref_runq_argmax(
        lg.ctypes.data_as(oracle.C.POINTER(oracle.C.c_float)), lg.size))
    if pos + 1 >= len(prompt):
        ids.append(tok)
print(({npos} - 1) / (time.perf_counter() - t0))
print(",".join(map(str, ids)))
"""
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        raise RuntimeError("reference runq failed: " + r.stderr[-500:])
    out = r.stdout.strip().splitlines()
    return float(out[0]), [int(t) for t in out[1].split(",") if t]


def runq_results(args):
    """Configs 1 and 2: runq.c's int8 models (stories15M / stories110M architectures, synthetic seeded weights,
    group size --gs (32, as the configs state; 64 is what tools/bin2q80.py gives stories110M), shared classifier)
    decoded on the device (mvb_runq_load + the captured step graph). One step = the rest
    of a 256-position run after the 4-token prompt (253 greedy tokens, positions 3 .. 255).
      value        device time of K steps (rewind to position 3 + 253 graph launches), L2 warm: the model is smaller
                   than the 126 MB L2, so a token's weights mostly stay there between tokens, as in a real decode
      flushed      the same tokens timed one by one with a 256 MB L2 flush before each (outside the timed events)
      e2e          mvb_runq_generate through the public API: prompt up, 253 ids back, host wall clock
      cpu_baseline runq.c's CPU build on the same file and prompt, all host cores, 64 positions"""
    import numpy as np
    import torch
    torch.cuda.set_device(0)
    mvb = load_pkg()
    sys.path.insert(0, PKG)
    import qwb
    names = [args.model] if args.model else list(RUNQ_MODELS)
    peak, peak_kind = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    lines = []
    for name in names:
        cfg_name, arch = RUNQ_MODELS[name]
        cfg = getattr(qwb, cfg_name)
        gs = args.gs
        path = os.path.join(DATA, f"{name}_g{gs}_s3.bin")
        if not os.path.exists(path):
            os.makedirs(DATA, exist_ok=True)
            qwb.write_synthetic_runq(path + ".tmp", cfg, seed=3, gs=gs)
            os.replace(path + ".tmp", path)
        prompt = [int(t) for t in np.random.default_rng(4).integers(3, cfg["vocab_size"], RUNQ_PROMPT)]
        npos = 256
        gen = npos - RUNQ_PROMPT + 1
        t0 = time.perf_counter()
        dec = mvb.RunqDecoder(path, ctx=cfg["seq_len"])
        load_s = time.perf_counter() - t0
        stream = torch.cuda.ExternalStream(dec.stream_handle)
        pos0, tok0 = RUNQ_PROMPT - 1, prompt[-1]
        dec.prefill(prompt)
        ids_ref = dec.decode(gen)

        def steps(k):
            for _ in range(k):
                dec.rewind(tok0, pos0, RUNQ_PROMPT)
                dec.launch(gen)
        steps(args.warmup)
        torch.cuda.synchronize()
        clocks = Clocks(0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        steps(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        t_dev = e0.elapsed_time(e1) / 1000.0
        value = args.steps * gen / t_dev
        # flushed: token by token, an L2-sized write before each (on the model's stream, outside the events)
        dec.rewind(tok0, pos0, RUNQ_PROMPT)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(gen)]
        with torch.cuda.stream(stream):
            for a, b in ev:
                flush.fill_(1)
                a.record(stream)
                dec.launch(1)
                b.record(stream)
        torch.cuda.synchronize()
        t_flush = sum(a.elapsed_time(b) for a, b in ev) / 1000.0
        # e2e through the public API
        ts = []
        for _ in range(max(1, min(args.steps, 5))):
            t0 = time.perf_counter()
            ids = dec.generate(prompt, gen)
            ts.append(time.perf_counter() - t0)
        t_e2e = statistics.median(ts)
        stop = ids_ref.tolist().index(1) if 1 in ids_ref.tolist() else gen
        if ids.tolist() != ids_ref.tolist()[:stop]:
            raise RuntimeError("generate disagrees with the decode steps")
        roof = step_roofline(dec, int(ids_ref[gen // 2 - 1]), pos0 + gen // 2, traffic=False)
        kernels = dec.cfg["kernels_per_step"]
        dec.close()
        cpu = None
        if not args.no_cpu_baseline and os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_runq.so")):
            threads = os.cpu_count()
            sample_pos = 64
            tps, ref_ids = run_reference_runq(path, prompt, sample_pos, threads)
            cpu = {"value": round(tps, 2), "unit": "tok/s", "cores": threads, "kind": "reference",
                   "sample": f"runq.c CPU build (-O3 -fopenmp -ffp-contract=off) forward() on the same file and "
                             f"prompt, {sample_pos} positions, tok/s from the end of the first forward as runq.c "
                             f"reports it",
                   "same_ids_as_b200": ref_ids == ids_ref.tolist()[:len(ref_ids)]}
        line = {"mode": "runq", "metric": f"runq int8 decode tok/s ({arch} arch, 1 B200)", "value": round(value, 1),
                "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1000.0 * t_dev / args.steps, 4),
                "us_per_token": round(1e6 * t_dev / args.steps / gen, 2),
                "higher_is_better": True, "dtype": "int8->int32, fp32", "data": "synthetic",
                "config": {"workload": f"{arch} architecture via runq (synthetic seeded runq v2 Q8_0, gs {gs}, shared "
                                       f"classifier), 4-token prompt, {gen} greedy tokens per step", "model": cfg,
                           "l2": "warm (weights fit in the 126 MB L2); 'flushed' gives the L2-flushed figure"},
                "flushed": {"value": round(gen / t_flush, 1), "unit": "tok/s",
                            "how": "each token timed alone after a 256 MB write to a scratch buffer"},
                "e2e": {"value": round(gen / t_e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * RUNQ_PROMPT + 32,
                        "d2h_bytes_per_step": 4 * gen + 32, "includes": "prompt feed (3 positions)"},
                "roofline": roof, "cpu_baseline": cpu, "gpu_launches": args.steps * gen * kernels,
                "kernels_per_token": kernels, "load_s": round(load_s, 3), "clocks": clk}
        lines.append(line)
    return lines


def runq_mode(args):
    for line in runq_results(args):
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="decode: leave out the sharded (config 5) block")
    ap.add_argument("--no-extra", action="store_true",
                    help="decode: leave out the runq (configs 1-2), sweep and prefill_gemm (config 4) blocks")
    ap.add_argument("--only", default="", help="sweep, prefill: run only this shape, rows x columns (e.g. 4864x896); "
                                               "prefill also takes any shape, Q4 unless qN follows (8192x8192, 65536x896q8)")
    ap.add_argument("--m", type=int, default=0, help="prefill: run only this token count")
    ap.add_argument("--model", default="", choices=["", *RUNQ_MODELS], help="runq: only this model")
    ap.add_argument("--full-head", action="store_true", help="step: the full-vocabulary head (mvb_qwen_full_head)")
    ap.add_argument("--gs", type=int, default=32, choices=[32, 64], help="runq: group size of the checkpoint")
    ap.add_argument("--mode", default="decode",
                    choices=["decode", "sweep", "sharded", "prefill", "prompt", "step", "runq"],
                    help="decode (the benchmark line), sweep (isolated matvec shapes), sharded (row-sharded matvec), "
                         "prefill (tensor-core matmul over many tokens), prompt (batched prompt prefill), "
                         "step (single decode steps), runq (configs 1 and 2: stories15M / stories110M decode)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.mode == "sweep":
            if rank == 0:
                reference_sweep(args)
            return
        reference_arm(args, rank, world)
        return
    if args.mode == "sweep":
        sweep_mode(args)
        return
    if args.mode == "prefill":
        prefill_mode(args)
        return
    if args.mode == "prompt":
        prompt_mode(args)
        return
    if args.mode == "step":
        step_mode(args)
        return
    if args.mode == "runq":
        runq_mode(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.mode == "sharded":
            if world == 1:
                import datetime
                import torch
                import torch.distributed as dist
                dist.init_process_group("gloo" if not torch.cuda.is_available() else "nccl", rank=0, world_size=1,
                                        init_method="tcp://127.0.0.1:29531", timeout=datetime.timedelta(seconds=120))
                world = 1
            sharded_mode(args, rank, world, local_rank)
        else:
            our_arm(args, rank, world, local_rank)
    finally:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
