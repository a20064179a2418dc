#!/usr/bin/env python
"""Benchmark of the B200 quantized matvec path.

Headline workload (one "step" = one sampler token): the Q6_K vocabulary
output projection 152064 x 3584 of a seeded synthetic hidden state, followed
by greedy argmax.  Rows are sharded over the ranks: rank r owns rows
[r*ceil(N/W), min(N, (r+1)*ceil(N/W))), runs the fused projection+argmax
kernel on its slice, and one NCCL all-gather joins every rank's logit slice
together with its 8-byte argmax key; the token is the maximum key.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Metric: algorithmic GB/s (packed weight bytes + f32 x + f32 logits per step,
whole job) over the timed steps, max over ranks of CUDA-event time.  Extra
keys: tokens/s, the kernel roofline, an end-to-end figure through the C ABI
with host buffers, the reference's CPU path on the host cores, and (N=1) the
other benchmark configurations.
"""
from __future__ import annotations

import argparse
import csv
import datetime
import importlib.util
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "my-inference-engine_b200")
Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14
VOCAB_ROWS, HIDDEN = 152064, 3584
METRIC = "Q4_K/Q6_K/Q8_0 GEMV weight GB/s vs HBM peak; decode tokens/s at 1/2/4/8 GPU"


def _load(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_qmv():
    build = _load("qmv_build", os.path.join(PKG, "build.py"))
    if not os.path.exists(build.LIB_PATH):
        build.build_library()
    mod = _load("my_inference_engine_b200", os.path.join(PKG, "__init__.py"))
    mod.load_library()
    return mod


def workloads():
    return _load("qmv_workloads", os.path.join(PKG, "workloads.py"))


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s of this pool's B200s (burst, cuBLAS) and its source."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def profile_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt,
    line 'dram_bytes_per_launch: <int>'), scaled by the caller; None if absent."""
    path = os.path.join(REPO, "profiles", name + ".txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples of this GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str | None):
        self.uuid = device_uuid
        self.proc = None
        self.out = None
        self.t0 = self.t1 = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu=timestamp,{self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "100"]
        if self.uuid:
            cmd[1:1] = ["-i", self.uuid]
        try:
            self.out = open("/tmp/qmv_clocks_%d.csv" % os.getpid(), "w+")
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def mark(self, which):
        setattr(self, which, datetime.datetime.now())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        rows = list(csv.reader(io.StringIO(self.out.read())))
        self.out.close()
        try:
            os.unlink(self.out.name)
        except OSError:
            pass
        samples, nearest = [], []
        for r in rows:
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                continue
            rec = {"ts": ts, "sm": float(r[2]), "max": float(r[3]), "power": r[4].strip(),
                   "hw_slowdown": r[6].strip(), "hw_thermal": r[7].strip(), "sw_thermal": r[8].strip(),
                   "sw_power_cap": r[9].strip()}
            nearest.append(rec)
            if self.t0 and self.t1 and self.t0 <= ts <= self.t1:
                samples.append(rec)
        used = samples
        note = None
        if not used and nearest and self.t0 and self.t1:
            mid = self.t0 + (self.t1 - self.t0) / 2
            used = sorted(nearest, key=lambda r: abs((r["ts"] - mid).total_seconds()))[:2]
            note = "timed region shorter than the sampling period: nearest samples used"
        if not used:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        reasons = []
        for key, label in (("hw_slowdown", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                           ("sw_thermal", "sw_thermal_slowdown"), ("sw_power_cap", "sw_power_cap")):
            if any(r[key] == "Active" for r in used):
                reasons.append(label)
        out = {"sm_mhz": statistics.median(r["sm"] for r in used), "sm_max_mhz": used[0]["max"],
               "reasons": reasons, "samples": len(used)}
        if note:
            out["note"] = note
        return out


# ------------------------------------------------------------ CPU reference

def cpu_reference_lib():
    """(Reference, kind): the reference's own OpenMP build (oracle/_ref) when
    present, else the scalar C restatement of it (a single-thread port)."""
    binding = _load("qmv_oracle_binding", os.path.join(REPO, "oracle", "binding.py"))
    if not os.path.exists(binding.REF_AVX2_SO) and os.path.isdir(os.path.join(binding.REFERENCE_SRC, "src")):
        binding.build(reference=True)
    if os.path.exists(binding.REF_AVX2_SO):
        return binding.Reference(binding.REF_AVX2_SO), "reference"
    if not os.path.exists(binding.ORACLE_SO):
        binding.build(reference=False)
    return binding.Oracle(), "port"


def cpu_vocab_step(lib, kind, blocks, x, threads):
    if kind == "reference":
        y = lib.matvec(Q6_K, blocks, VOCAB_ROWS, HIDDEN, x)
        ok, tok, _ = lib.greedy(y)
    else:
        y = lib.matvec(Q6_K, blocks, VOCAB_ROWS, HIDDEN, x, threads=threads)
        ok, tok = lib.argmax(y)
    return tok


def reference_vocab_logits(x, cores):
    """Configuration 2 on the host, as the parity gate's reference: the
    reference's own scalar build (oracle/_ref, its src/quantized_matvec.cpp
    projection and src/sampler.cpp greedy sampler; the C restatement when that
    build is absent) on the full seeded 152064 x 3584 matrix.  Returns
    (logits f32, per-row tolerance 1e-4 * sum|w x| f64, token, source)."""
    binding = _load("qmv_oracle_binding", os.path.join(REPO, "oracle", "binding.py"))
    wl = workloads()
    blocks = wl.make_blocks(Q6_K, VOCAB_ROWS, HIDDEN, seed=0)
    oracle = binding.Oracle()
    if os.path.exists(binding.REF_SCALAR_SO):
        ref = binding.Reference(binding.REF_SCALAR_SO)
        ref.set_threads(cores)
        y_ref = ref.matvec(Q6_K, blocks, VOCAB_ROWS, HIDDEN, x)
        ok, tok, _ = ref.greedy(y_ref)
        source = "reference scalar build (oracle/_ref: src/quantized_matvec.cpp + src/sampler.cpp)"
    else:
        y_ref = oracle.matvec(Q6_K, blocks, VOCAB_ROWS, HIDDEN, x, threads=cores)
        ok, tok = oracle.argmax(y_ref)
        source = "C restatement of the reference's scalar path (oracle/qmv_oracle.c)"
    bound = 1e-4 * oracle.row_abs_dot(Q6_K, blocks, VOCAB_ROWS, HIDDEN, x, threads=cores)
    return y_ref, bound, (tok if ok else -1), source


def check_vocab_parity(logits, token, x, dev, rank, world):
    """Every rank compares its full gathered logits and its global token with
    the reference's (computed once on rank 0 and broadcast).  Returns the
    parity record (rank 0: the worst rank's figures) and whether it passed."""
    import torch
    import torch.distributed as dist
    if rank == 0:
        y_ref, bound, ref_tok, source = reference_vocab_logits(x, os.cpu_count() or 1)
        t_ref = torch.from_numpy(y_ref).to(dev)
        t_bound = torch.from_numpy(bound).to(dev)
        t_tok = torch.tensor([ref_tok], dtype=torch.int64, device=dev)
    else:
        t_ref = torch.empty(VOCAB_ROWS, dtype=torch.float32, device=dev)
        t_bound = torch.empty(VOCAB_ROWS, dtype=torch.float64, device=dev)
        t_tok = torch.empty(1, dtype=torch.int64, device=dev)
        source = None
    if world > 1:
        for t in (t_ref, t_bound, t_tok):
            dist.broadcast(t, 0)
    y_ref = t_ref.cpu().numpy()
    bound = t_bound.cpu().numpy()
    ref_tok = int(t_tok.item())
    err = np.abs(logits.astype(np.float64) - y_ref.astype(np.float64))
    ratio = float(np.max(err / np.maximum(bound, 1e-300)))
    rows_out = int(np.count_nonzero(err > bound))
    match = 1.0 if (token == ref_tok and ref_tok >= 0) else 0.0
    agg = torch.tensor([ratio, float(rows_out), -match], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(agg, op=dist.ReduceOp.MAX)
    ratio, rows_out, match = float(agg[0]), int(agg[1]), -float(agg[2])
    top2 = np.sort(y_ref)[-2:]
    rec = {"token": token, "reference_token": ref_tok, "token_match": match == 1.0,
           "max_err_over_bound": round(ratio, 5), "rows_out_of_bound": rows_out,
           "rows_checked": VOCAB_ROWS, "ranks_checked": world, "seed": 0,
           "reference_top2_gap": float(top2[1] - top2[0]), "reference": source,
           "bound": "|y - y_ref| <= 1e-4 * sum|w x| per row; identical greedy token"}
    return rec, (match == 1.0 and ratio <= 1.0)


def time_cpu_reference(blocks, x, min_seconds, max_steps=None):
    lib, kind = cpu_reference_lib()
    cores = os.cpu_count() or 1
    if kind == "reference":
        lib.set_threads(cores)
    cpu_vocab_step(lib, kind, blocks, x, cores)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_vocab_step(lib, kind, blocks, x, cores)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or (max_steps and n >= max_steps):
            break
    return n, el, kind, cores


# --------------------------------------------------------------- helpers

def vocab_bytes(rows):
    return rows * (HIDDEN // 256) * 210


def bench_config(world):
    """The workload both arms report (identical keys and values for one N)."""
    return {"workload": "cfg2_q6_k_vocab_projection_argmax", "rows": VOCAB_ROWS, "cols": HIDDEN,
            "ggml_type": "Q6_K", "parallelism": f"row-shard x{world}",
            "rows_per_rank": -(-VOCAB_ROWS // world),
            "l2_defeat": "inputs larger than L2: 447 MB of weights per step at N=1; at N>1 each rank "
                         "rotates over weight copies of its shard totalling >= 2.5x L2"}


def shard(rank, world):
    per = -(-VOCAB_ROWS // world)
    b = min(VOCAB_ROWS, rank * per)
    e = min(VOCAB_ROWS, (rank + 1) * per)
    return b, e, per


def copies_for(slice_bytes, l2_bytes):
    """Distinct weight copies so the rotating set is >= 2.5x L2 (no L2 reuse
    between consecutive launches)."""
    return max(1, math.ceil(2.5 * l2_bytes / max(1, slice_bytes)))


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    wl = workloads()
    blocks = wl.make_blocks(Q6_K, VOCAB_ROWS, HIDDEN, seed=0)
    x = wl.make_activations(HIDDEN, seed=0)
    lib, kind = cpu_reference_lib()
    cores = os.cpu_count() or 1
    if kind == "reference":
        lib.set_threads(cores)
    for _ in range(args.warmup):
        cpu_vocab_step(lib, kind, blocks, x, cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_vocab_step(lib, kind, blocks, x, cores)
    el = time.perf_counter() - t0
    step_bytes = vocab_bytes(VOCAB_ROWS) + 4 * HIDDEN + 4 * VOCAB_ROWS
    value = args.steps * step_bytes / el / 1e9
    sample = f"full {VOCAB_ROWS}x{HIDDEN} Q6_K projection + greedy argmax per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * el / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tokens_per_s": round(args.steps / el, 3),
        "config": bench_config(world),
        "implementation": {"step": "the reference's quantized_tensor_matvec_f32 + sampler_greedy_sample "
                                   "(OpenMP over rows on the host cores)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- b200 arm

def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    qmv = load_qmv()
    qmv.set_device(local_rank)
    sh = _load("qmv_sharding", os.path.join(PKG, "sharding.py"))
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    props = torch.cuda.get_device_properties(local_rank)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    wl = workloads()
    p2p = world > 1 and args.exchange == "p2p"

    b, e, per = sh.shard_rows(VOCAB_ROWS, world, rank)
    rows = e - b
    blocks = wl.make_blocks(Q6_K, VOCAB_ROWS, HIDDEN, seed=0, row_begin=b, row_end=e)
    copies = copies_for(vocab_bytes(rows), l2)
    weights = [qmv.Weight.from_row_slice(Q6_K, blocks, VOCAB_ROWS, HIDDEN, b) for _ in range(copies)]
    del blocks
    x_host = wl.make_activations(HIDDEN, seed=0)
    x_dev = torch.from_numpy(x_host).to(dev)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    # NCCL mode: one all-gather of {logit slice, 8-byte key} per rank
    per_pad = (per + 3) // 4 * 4
    stride = per_pad + 2
    sendbuf = torch.zeros(stride, dtype=torch.float32, device=dev)
    gathered = torch.zeros(world * stride, dtype=torch.float32, device=dev)
    keyview = sendbuf[per_pad:per_pad + 2].view(torch.int64)
    SIGN = torch.tensor(-(1 << 63), dtype=torch.int64, device=dev)
    # p2p mode: fused kernel, exchange over peer memory
    group = sh.ExchangeGroup(qmv, rank, world, per) if p2p else None
    gkey = torch.zeros(1, dtype=torch.int64, device=dev)

    def global_key():
        if p2p:
            return int(gkey.item()) & 0xFFFFFFFFFFFFFFFF
        if world > 1:
            keys = gathered.view(world, stride)[:, per_pad:per_pad + 2].contiguous().view(torch.int64).view(-1)
            return int(torch.bitwise_xor(torch.bitwise_xor(keys, SIGN).max(), SIGN).item()) & 0xFFFFFFFFFFFFFFFF
        return int(keyview.item()) & 0xFFFFFFFFFFFFFFFF

    kstart = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kend = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    def launch(i, sp):
        """One step's kernel (plus the NCCL all-gather in NCCL mode) on stream sp."""
        w = weights[i % copies]
        if p2p:
            group.next_epoch()
            w.matvec_argmax_exchange(x_dev.data_ptr(), rank, world, group.buffers, per, gkey.data_ptr(),
                                     ws.data_ptr(), sp)
        else:
            w.matvec_argmax(x_dev.data_ptr(), sendbuf.data_ptr(), keyview.data_ptr(), ws.data_ptr(), sp)

    def step(i, timed):
        if timed:
            kstart[i].record(stream)
        launch(i, sptr)
        if timed:
            kend[i].record(stream)
        if world > 1 and not p2p:
            dist.all_gather_into_tensor(gathered, sendbuf)

    def gathered_logits():
        """This rank's copy of all VOCAB_ROWS logits of the latest step."""
        if world == 1:
            return sendbuf[:rows].cpu().numpy()
        if p2p:
            host = np.empty(world * per, np.float32)
            qmv.memcpy(host, qmv.exchange_logits(group.own, world, per, group.epoch), host.nbytes, sptr)
        else:
            host = gathered.view(world, stride)[:, :per].contiguous().view(-1).cpu().numpy()
        return np.concatenate([host[s0:s1] for s0, s1 in sh.gathered_rows(VOCAB_ROWS, world)])

    # correctness gate before timing (seed 0): every rank's full logits and
    # its global token against the reference's own scalar build
    step(0, False)
    torch.cuda.synchronize()
    token = qmv.key_to_token(global_key())
    parity, parity_ok = check_vocab_parity(gathered_logits(), token, x_host, dev, rank, world)
    if not parity_ok:
        for wobj in weights:
            wobj.free()
        if world > 1:
            dist.barrier()
            if group is not None:
                group.close()
            dist.destroy_process_group()
        if rank == 0:
            return {"metric": METRIC, "error": "parity gate failed on configuration 2", "parity": parity,
                    "n_gpus": world, "config": bench_config(world)}, False
        return None, False

    for i in range(args.warmup):
        step(i, False)
    uuid = None
    try:
        uuid = "GPU-" + str(props.uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid) if rank == 0 else None
    if clocks:
        clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    # The K timed steps are replayed from one CUDA graph when the step is our
    # kernel alone (N = 1, or the fused peer exchange), so launch overhead is
    # not timed; NCCL mode launches step by step.
    use_graph = world == 1 or p2p
    graph = None
    if use_graph:
        gstream = torch.cuda.Stream(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gstream):
            for i in range(args.steps):
                launch(i, gstream.cuda_stream)
        with torch.cuda.stream(gstream):
            graph.replay()  # untimed replay (warm-up of the graph itself)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    if clocks:
        clocks.mark("t0")
    if use_graph:
        with torch.cuda.stream(gstream):
            t_start.record(gstream)
            graph.replay()
            t_end.record(gstream)
    else:
        t_start.record(stream)
        for i in range(args.steps):
            step(i, True)
        t_end.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark("t1")
    if world > 1:
        dist.barrier()
    ms = t_start.elapsed_time(t_end)
    if use_graph:
        kms = ms / args.steps  # the graph holds only the kernels
        if p2p:
            # capture advanced the host count once; each replay advanced the device count again
            group.next_epoch(args.steps)
    else:
        kms = sum(kstart[i].elapsed_time(kend[i]) for i in range(args.steps)) / args.steps
    del graph
    t = torch.tensor([ms, kms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kms_max = float(t[0]), float(t[1])
    clock_info = clocks.stop() if clocks else None

    # N > 1: the same shard projection + argmax without any exchange (each
    # rank alone, graph-replayed), so the step splits into shard compute and
    # the cost of joining the ranks (exchange stores, flags, waiting for the
    # slowest rank; in NCCL mode the all-gather)
    breakdown = None
    if world > 1:
        g2 = torch.cuda.CUDAGraph()
        gs2 = torch.cuda.Stream(dev)
        with torch.cuda.graph(g2, stream=gs2):
            for i in range(args.steps):
                weights[i % copies].matvec_argmax(x_dev.data_ptr(), sendbuf.data_ptr(), keyview.data_ptr(),
                                                  ws.data_ptr(), gs2.cuda_stream)
        with torch.cuda.stream(gs2):
            g2.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(gs2):
            a2.record(gs2)
            g2.replay()
            b2.record(gs2)
        torch.cuda.synchronize()
        del g2
        tb = torch.tensor([a2.elapsed_time(b2) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(tb, op=dist.ReduceOp.MAX)
        shard_us = float(tb[0]) * 1e3
        step_us = ms / args.steps * 1e3
        breakdown = {
            "step_us": round(step_us, 2),
            "shard_projection_argmax_us": round(shard_us, 2),
            "join_us": round(step_us - shard_us, 2),
            "join": ("fused exchange: logit stores to peers, flags, the wait for the slowest rank"
                     if p2p else "NCCL all-gather of logit slices and keys, launched after each kernel"),
            "nvlink_bytes_per_step_per_rank": (4 * per + 8 + 4) * (world - 1),
            "shard_bytes_per_step": vocab_bytes(rows) + 4 * HIDDEN + 4 * rows,
            "shard_roofline_us": round((vocab_bytes(rows) + 4 * HIDDEN + 4 * rows) / (measured_peaks()[0] * 1e3), 2),
        }
        if not p2p:
            breakdown["kernel_us_events"] = round(kms_max * 1e3, 2)

    # ---- end to end through the C ABI with host buffers (pinned)
    x_pin = torch.from_numpy(x_host).pin_memory()
    out_floats = world * per if p2p else world * stride
    out_pin = torch.empty(out_floats, dtype=torch.float32).pin_memory()
    key_pin = torch.empty(1, dtype=torch.int64).pin_memory()
    e2e_steps = max(3, min(args.steps, 200))

    def e2e_step(i):
        x_dev.copy_(x_pin, non_blocking=True)
        step(i, False)
        if rank == 0:
            if p2p:
                key_pin.copy_(gkey, non_blocking=True)
                # gathered logits, out of the library-owned exchange buffer (same stream)
                qmv.memcpy(out_pin.data_ptr(), qmv.exchange_logits(group.own, world, per, group.epoch),
                           4 * out_floats, sptr)
            elif world > 1:
                out_pin.copy_(gathered, non_blocking=True)
            else:
                out_pin[:stride].copy_(sendbuf, non_blocking=True)
        stream.synchronize()
        if rank == 0:
            if p2p:
                return qmv.key_to_token(int(key_pin.numpy().view(np.uint64)[0]))
            keys = out_pin.numpy().reshape(world, stride)[:, per_pad:per_pad + 2].copy().view(np.uint64)
            return qmv.key_to_token(int(keys.max()))
        return None

    for i in range(2):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_tok = None
    for i in range(e2e_steps):
        e2e_tok = e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms[0])
    status = qmv.device_status()

    step_bytes = vocab_bytes(VOCAB_ROWS) + world * 4 * HIDDEN + 4 * VOCAB_ROWS
    value = args.steps * step_bytes / (ms * 1e-3) / 1e9
    e2e_value = e2e_steps * step_bytes / (e2e_ms * 1e-3) / 1e9

    result = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        launch_bytes = vocab_bytes(rows) + 4 * HIDDEN + 4 * rows
        achieved = launch_bytes / (kms_max * 1e-3) / 1e9
        traffic = profile_traffic("gemv_q6_k_cfg2")
        if traffic is not None:
            traffic = traffic * rows / VOCAB_ROWS
        if world == 1:
            par = "row-shard x1"
        elif p2p:
            par = f"row-shard x{world}, fused exchange over peer memory (NVLink)"
        else:
            par = f"row-shard x{world} + NCCL all-gather"
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-dp4a/f32",
            "data": "synthetic (seeded splitmix64; Q6_K blocks per the configuration)",
            "tokens_per_s": round(args.steps / (ms * 1e-3), 1),
            "token": token,
            "parity": parity,
            "config": bench_config(world),
            "implementation": {"step": par, "weight_copies_per_rank": copies},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "gemv_tma_kernel<Q6_K> fused argmax" + (" + exchange" if p2p else ""),
                         "kernel_ms": round(kms_max, 5), "peak_source": peak_kind},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * HIDDEN,
                    "d2h_bytes_per_step": 4 * out_floats + (8 if p2p else 0), "steps": e2e_steps,
                    "tokens_per_s": round(e2e_steps / (e2e_ms * 1e-3), 1), "token": e2e_tok,
                    "token_matches_reference": e2e_tok == parity["reference_token"]},
            "gpu_launches": args.steps,
            "breakdown": breakdown,
            "clocks": clock_info,
            "device_status": status,
        }
    for wobj in weights:
        wobj.free()
    del weights
    if world > 1:
        dist.barrier()
        if group is not None:
            group.close()
        dist.destroy_process_group()
    return result, True


SECONDARY = (("cfg0_q8_0_4864x896", 0), ("cfg1a_q4_k_18944x3584", 0), ("cfg1b_q4_k_3584x18944", 0),
             ("cfg3_q5_0_4864x896", 8), ("cfg3_q5_0_4864x896", 512))


def extras_single_gpu(qmv, steps, only=None):
    """Secondary configurations on one GPU: per call, algorithmic GB/s (and
    TFLOP/s for batched calls).  The calls rotate over enough weight copies to
    exceed 2.5x L2 and are replayed from a CUDA graph, so the figure is device
    time, not Python launch overhead."""
    import torch
    wl = workloads()
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    peak, _ = measured_peaks()
    out = {}
    for name, batch in SECONDARY:
        key = name if not batch else f"{name}_P{batch}"
        if only and key != only:
            continue
        gtype, rows, cols = wl.CONFIGS[name]
        blocks = wl.make_blocks(gtype, rows, cols, seed=0)
        copies = copies_for(blocks.nbytes, l2)
        ws = [qmv.Weight(gtype, blocks, rows, cols) for _ in range(copies)]
        P = max(1, batch)
        X = torch.from_numpy(np.stack([wl.make_activations(cols, seed=p) for p in range(P)])).cuda()
        Y = torch.empty((P, rows), dtype=torch.float32, device="cuda")
        n = max(steps, copies)
        stream = torch.cuda.Stream()

        def call(i):
            sp = stream.cuda_stream
            if batch:
                ws[i % copies].matmul(X.data_ptr(), P, Y.data_ptr(), sp)
            else:
                ws[i % copies].matvec(X.data_ptr(), Y.data_ptr(), sp)

        with torch.cuda.stream(stream):
            for i in range(3 * copies):
                call(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n):
                call(i)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):  # replay and both events on one stream
            graph.replay()
            torch.cuda.synchronize()
            a.record(stream)
            graph.replay()
            b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        alg = wl.algorithmic_bytes(gtype, rows, cols, P)
        rec = {"us_per_call": round(ms * 1e3, 2), "GB_s": round(alg / (ms * 1e-3) / 1e9, 1),
               "frac_hbm": round(alg / (ms * 1e-3) / 1e9 / peak, 3), "copies": copies, "calls": n,
               "timing": "CUDA graph replay"}
        if batch:
            tflops = 2.0 * P * rows * cols / (ms * 1e-3) / 1e12
            rec["TFLOP_s"] = round(tflops, 2)
            if P >= 32:
                # tensor-core kernel: three bf16 MMAs per product (wh*xh + wl*xh + wh*xl)
                tpeak, tkind = measured_tensor_peak()
                rec["kernel"] = "matmul_tc_kernel (tcgen05.mma kind::f16, bf16 hi/lo splits)"
                rec["tensor_TFLOP_s_issued"] = round(3 * tflops, 2)
                rec["frac_tensor"] = round(3 * tflops / tpeak, 3)
                rec["tensor_peak_source"] = tkind
        out[key] = rec
        del graph
        for w in ws:
            w.free()
    return out


QWEN2_DECODE = "cfg4_qwen2_0_5b_decode"


def qwen2_free_run(binding, m, tensors, max_ctx, keys, vals, gpu_tokens, seconds):
    """Free-run token identity of configuration 4: the reference's own scalar
    build (oracle/_ref: forward_token, src/qwen2_architecture.cpp:1195-1531,
    then sampler_greedy_sample, src/sampler.cpp:14-36) decodes greedily from
    the same cache and start token, feeding back its own tokens, until its
    token differs from the GPU's, all GPU tokens are compared, or `seconds`
    pass.  At a divergence the reference's logit gap between its token and the
    GPU's says whether the two were a near tie."""
    ref = binding.RefQwen2(m, tensors, max_ctx, path=binding.REF_SCALAR_SO)
    sampler = binding.Reference(binding.REF_SCALAR_SO)
    first, n, tok = None, 0, 7
    t0 = time.perf_counter()
    try:
        ref.set_kv(keys, vals)
        for i in range(len(gpu_tokens)):
            ok, logits = ref.forward(tok)
            ok2, rtok, _ = sampler.greedy(logits)
            if not (ok and ok2):
                first = {"step": i, "reference_failed": True}
                break
            g = int(gpu_tokens[i])
            if rtok != g:
                gap = float(logits[rtok]) - float(logits[g]) if 0 <= g < logits.size else None
                first = {"step": i, "gpu_token": g, "reference_token": int(rtok), "reference_logit_gap": gap,
                         "gap_over_max_abs_logit": (gap / float(np.max(np.abs(logits)))) if gap is not None else None}
                break
            n += 1
            tok = rtok
            if time.perf_counter() - t0 > seconds:
                break
    finally:
        ref.close()
    return {"gpu_tokens": len(gpu_tokens), "compared": n + (1 if first else 0), "identical": n,
            "first_divergence": first, "seconds": round(time.perf_counter() - t0, 1),
            "reference": "the reference's scalar build (forward_token + sampler_greedy_sample), "
                         "feeding back its own tokens from the same 1024-position cache and start token 7"}


def bench_qwen2_decode(qmv, steps=256, prefill=1024, cpu_seconds=5.0, cpu=True, free_seconds=45.0):
    """Configuration 4: greedy decode of `steps` tokens on the synthetic
    Qwen2-0.5B model from a KV cache pre-filled to `prefill` positions.
    value: device-timed tokens/s (CUDA events around `steps` replays of the
    step graph on one stream; the token is fed back on the device).  e2e:
    qmv_qwen2_generate through the C ABI (first token in, `steps` ids out),
    wall clock.  Bytes per token: packed weights of every layer and of the
    output projection, the embedding row, and the KV cache read by attention."""
    import torch
    wl = workloads()
    m = wl.make_qwen2("cfg4_qwen2_0_5b", seed=0)
    tensors = wl.qwen2_tensor_list(m)
    keys, vals = wl.make_kv_cache(m, prefill, seed=0)
    max_ctx = prefill + steps
    dec = qmv.Qwen2Decoder(m, tensors, max_ctx)
    try:
        stream = torch.cuda.Stream()
        dec.set_kv(keys, vals)
        dec.generate(7, min(8, steps))  # warm-up (within the steps the context holds)
        dec.set_kv(keys, vals)
        dec.begin(7)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            a.record(stream)
            dec.replay(steps, stream.cuda_stream)
            b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        toks, pos = dec.read(steps)
        dec.set_kv(keys, vals)
        t0 = time.perf_counter()
        toks_e2e = dec.generate(7, steps)
        e2e_s = time.perf_counter() - t0
        status = qmv.device_status(clear=True)
        launches = dec.kernels_per_step
    finally:
        dec.close()
    packed = sum(t[4].nbytes for t in tensors if t[3] > 0 and t[0] != "token_embd.weight")
    embd_row = m["embd"][3].shape[1]
    kvd = m["kv_heads"] * (m["dim"] // m["heads"])
    kv_read = sum(2 * m["layers"] * (prefill + i + 1) * kvd * 4 for i in range(steps)) / steps
    per_token = packed + embd_row + kv_read
    peak, _ = measured_peaks()
    gbs = per_token * steps / (ms * 1e-3) / 1e9
    rec = {"tokens_per_s": round(steps / (ms * 1e-3), 1), "us_per_token": round(ms * 1e3 / steps, 2),
           "tokens": steps, "prefill": prefill, "bytes_per_token": int(per_token), "GB_s": round(gbs, 1),
           "frac_hbm": round(gbs / peak, 3),
           "gpu_launches_per_token": launches,
           "e2e": {"tokens_per_s": round(steps / e2e_s, 1), "h2d_bytes": 8, "d2h_bytes": 4 * steps},
           "same_tokens_e2e": bool(np.array_equal(toks, toks_e2e)), "next_position": pos,
           "timing": "CUDA events around graph replays (one stream)", "device_status": status,
           "model": "Qwen2-0.5B architecture, random-init (Q8_0 attention/gate/embedding/output, Q5_0 up/down)"}
    if cpu:
        binding = _load("qmv_oracle_binding", os.path.join(REPO, "oracle", "binding.py"))
        if os.path.exists(binding.REF_SCALAR_SO):
            rec["free_run"] = qwen2_free_run(binding, m, tensors, max_ctx, keys, vals, toks, free_seconds)
        if os.path.exists(binding.REF_AVX2_SO):
            ref = binding.RefQwen2(m, tensors, max_ctx, path=binding.REF_AVX2_SO)
            try:
                ref.set_kv(keys, vals)
                n, tok, t0 = 0, 7, time.perf_counter()
                while n < steps and (time.perf_counter() - t0) < cpu_seconds:
                    ok, logits = ref.forward(tok)
                    tok = int(np.argmax(logits))
                    n += 1
                el = time.perf_counter() - t0
            finally:
                ref.close()
            rec["cpu_baseline"] = {"value": round(n / el, 2), "unit": "tokens/s", "cores": os.cpu_count(),
                                   "kind": "reference",
                                   "sample": f"{n} decode steps from {prefill} cached positions "
                                             f"(reference forward_token, OpenMP AVX2 build, {el:.1f} s)"}
    return rec


QWEN2_PREFILL = "cfg4_qwen2_0_5b_prefill1024"


def bench_qwen2_prefill(qmv, prompt=1024, reps=5, cpu_seconds=5.0, cpu=True):
    """Time to first token on the configuration-4 model: a `prompt`-token
    prompt appended from position 0 through qmv_qwen2_prefill (every layer's
    projections as batched matmuls over the 1024 positions, causal attention,
    the last position's logits and greedy token).  value: prompt tokens per
    second of device time (CUDA events on the decoder's stream around the
    call); e2e: the same through the C ABI by wall clock, ids in and logits
    out.  FLOPs: 2 x positions x layer weights, the output projection for the
    last position, and 4 x heads x head_dim x visible keys per position and
    layer for attention."""
    import torch
    wl = workloads()
    m = wl.make_qwen2("cfg4_qwen2_0_5b", seed=0)
    tensors = wl.qwen2_tensor_list(m)
    ids = np.random.default_rng(0).integers(0, m["vocab"], prompt).astype(np.int32)
    dec = qmv.Qwen2Decoder(m, tensors, prompt + 8)
    dev_ms, wall_ms = [], []
    try:
        stream = torch.cuda.ExternalStream(dec.stream)
        for _ in range(2):  # warm-up (buffers, dynamic shared memory limits, memory pool)
            dec.reset()
            dec.prefill(ids)
        for _ in range(reps):
            dec.reset()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record(stream)
            t0 = time.perf_counter()
            _, tok = dec.prefill(ids)
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            b.record(stream)
            b.synchronize()
            dev_ms.append(a.elapsed_time(b))
        status = qmv.device_status(clear=True)
    finally:
        dec.close()
    layer_w = sum(t[2] * t[3] for t in tensors if t[3] > 0 and t[0].startswith("blk."))
    hd = m["dim"] // m["heads"]
    attn = 4 * m["heads"] * hd * m["layers"] * prompt * (prompt + 1) / 2
    flops = 2 * prompt * layer_w + 2 * m["vocab"] * m["dim"] + attn
    ms = float(np.median(dev_ms))
    peak, _ = measured_tensor_peak()
    rec = {"tokens_per_s": round(prompt / (ms * 1e-3), 1), "ms_per_prompt": round(ms, 3),
           "ms_min": round(min(dev_ms), 3), "prompt": prompt, "reps": reps,
           "TFLOP_s": round(flops / (ms * 1e-3) / 1e12, 1), "GFLOP_per_prompt": round(flops / 1e9, 1),
           "frac_tensor": round(flops / (ms * 1e-3) / 1e12 / peak, 3) if peak else None,
           "e2e": {"tokens_per_s": round(prompt / (float(np.median(wall_ms)) * 1e-3), 1),
                   "ms_per_prompt": round(float(np.median(wall_ms)), 3), "h2d_bytes": 4 * prompt,
                   "d2h_bytes": 4 * m["vocab"]},
           "next_token": tok, "device_status": status,
           "timing": "CUDA events on the decoder stream around qmv_qwen2_prefill (median of reps)",
           "model": "Qwen2-0.5B architecture, random-init (Q8_0 attention/gate/embedding/output, Q5_0 up/down)"}
    if cpu:
        binding = _load("qmv_oracle_binding", os.path.join(REPO, "oracle", "binding.py"))
        if os.path.exists(binding.REF_AVX2_SO):
            ref = binding.RefQwen2(m, tensors, prompt + 8, path=binding.REF_AVX2_SO)
            try:
                seg, n, t0 = 64, 0, time.perf_counter()
                ref.reset()
                while n + seg <= prompt and (time.perf_counter() - t0) < cpu_seconds:
                    ok, _ = ref.prefill(ids[n:n + seg])
                    assert ok
                    n += seg
                el = time.perf_counter() - t0
            finally:
                ref.close()
            rec["cpu_baseline"] = {"value": round(n / el, 2), "unit": "tokens/s", "cores": os.cpu_count(),
                                   "kind": "reference",
                                   "sample": f"the first {n} prompt tokens in {seg}-token prefill_tokens calls "
                                             f"(OpenMP AVX2 build, {el:.1f} s)"}
    return rec


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: fused peer-memory exchange (default) or a separate NCCL all-gather")
    ap.add_argument("--only", default=None,
                    help="run one secondary configuration only (e.g. cfg1a_q4_k_18944x3584, "
                         "cfg3_q5_0_4864x896_P512) for --steps calls; used for profiling")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(json.dumps({"error": "run N>1 under torchrun (one process per GPU)"}), flush=True)
        return 2
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.only:
        import torch
        torch.cuda.set_device(local_rank)
        qmv = load_qmv()
        qmv.set_device(local_rank)
        if args.only == QWEN2_DECODE:
            res = {QWEN2_DECODE: bench_qwen2_decode(qmv, steps=min(args.steps, 256), cpu=not args.no_cpu_baseline)}
        elif args.only == QWEN2_PREFILL:
            res = {QWEN2_PREFILL: bench_qwen2_prefill(qmv, cpu=not args.no_cpu_baseline)}
        else:
            res = extras_single_gpu(qmv, args.steps, args.only)
        print(json.dumps({"only": args.only, "result": res}), flush=True)
        return 0

    result, ok = run_b200(args, rank, world, local_rank)
    if not ok:
        if rank == 0:
            print(json.dumps(result), flush=True)
        return 3
    if rank != 0:
        return 0
    if world == 1 and not args.no_extras:
        qmv = load_qmv()
        result["configs"] = extras_single_gpu(qmv, steps=200)
        result["configs"][QWEN2_DECODE] = bench_qwen2_decode(qmv, cpu=not args.no_cpu_baseline)
        result["configs"][QWEN2_PREFILL] = bench_qwen2_prefill(qmv, cpu=not args.no_cpu_baseline)
    if world == 1 and not args.no_cpu_baseline:
        wl = workloads()
        blocks = wl.make_blocks(Q6_K, VOCAB_ROWS, HIDDEN, seed=0)
        x = wl.make_activations(HIDDEN, seed=0)
        n, el, kind, cores = time_cpu_reference(blocks, x, args.cpu_seconds)
        step_bytes = vocab_bytes(VOCAB_ROWS) + 4 * HIDDEN + 4 * VOCAB_ROWS
        result["cpu_baseline"] = {
            "value": round(n * step_bytes / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{n} full {VOCAB_ROWS}x{HIDDEN} Q6_K projections + greedy argmax "
                      f"({el:.1f} s, {'reference OpenMP AVX2 build' if kind == 'reference' else 'scalar C port'})"}
    print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
