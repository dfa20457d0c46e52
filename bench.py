#!/usr/bin/env python
"""Benchmark of B200 paged decode attention (xLLMs' decode hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c1|c3|c4|c5]

One step = one decode-attention pass over the whole batch (one new token per
sequence). N = 1 runs BASELINE config 2 (Llama-3-8B GQA, B = 64, fp16 KV,
context U[1024, 8192]). With N > 1 (launched by torch.distributed.run, one
rank per GPU) the batch grows to 64*N sequences and the 8 KV heads are
sharded over the ranks (KV-head-group sharding): per-GPU work stays that of
config 2 ("scaling": "weak"), each rank holds its own page pool and block
tables, and every rank's kernels store its heads' output rows into every
GPU's [B, Hq, D] buffer over NVLink (the fused head gather; --gather nccl
runs an NCCL all-gather + head interleave instead). --workload c5 is config 5
(B = 512 fixed, 64/8 heads, context U[4096, 16384]) split over the N GPUs
("scaling": "strong").

Every run checks its own output outside the timed regions: on each rank a
sample of sequences of the gathered [B, Hq, D] output is compared with the
CPU oracle over that rank's pools (its heads), and every rank's gathered
buffer must equal every other's bit for bit. The line carries parity_ok and
parity_worst; the process exits non-zero when the check fails.

Printed by rank 0: one JSON line. `value` is algorithmic GB/s of the whole
job (KV + Q + out + block tables + seq_lens) with inputs resident in HBM,
device-timed with CUDA events, max over ranks. `e2e` is the same metric
through the backend plugin's C ABI with Q / block tables / seq_lens copied
host->device and the output device->host inside every step (K steps
enqueued back to back; `e2e.host_synced` waits on the host for each step's
output before the next, as a decode loop does). `roofline` covers the
attention kernel alone (events recorded around it by the library);
`per_rank` splits a step into attention, merge and gather-barrier time on
every rank. `cpu_baseline` times the reference's CPU attention on the host.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "paged-decode KV-read GB/s (% of HBM peak) & seq-tokens/s at 1/2/4/8 GPU"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c5", "act"], default="c2",
                    help="c1..c5: the paged-attention configurations; act: one activation "
                         "operator (--act-op) on a Llama-3-8B MLP-sized input, 1 GPU")
    ap.add_argument("--graph", action="store_true",
                    help="1 GPU: capture one step in a CUDA graph and time K replays "
                         "(device time of launch-bound small configurations such as c1)")
    ap.add_argument("--kv", choices=["fp16", "e4m3", "e5m2", "int8"], default="fp16",
                    help="KV cache format (c2/c3/c5, 1 GPU): e4m3 / e5m2 = fp8 pools, int8 = "
                         "int8 pools, one scale per pool (nxt_paged_attention_fp8_ex)")
    ap.add_argument("--act-op", default="silu_and_mul",
                    choices=["silu_and_mul", "mul_and_silu", "gelu_and_mul",
                             "gelu_tanh_and_mul", "gelu", "silu"])
    ap.add_argument("--act-tokens", type=int, default=8192)
    ap.add_argument("--act-d", type=int, default=14336)
    ap.add_argument("--cpu-seconds", type=float, default=6.0,
                    help="wall-time budget of the cpu_baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the e2e leg (profiling runs)")
    ap.add_argument("--gather", choices=["fused", "fused-mc", "nccl"], default="fused",
                    help="N > 1: fused = kernels store each rank's heads into every GPU's "
                         "buffer over NVLink (nxt_paged_attention_sharded); fused-mc = the same "
                         "with one multimem (NVLS) store per row chunk into buffers from torch "
                         "symmetric memory; nccl = NCCL all-gather + head interleave")
    ap.add_argument("--prefix", choices=["on", "off"], default="on",
                    help="c4: on = shared-prefix (cascade) attention over the radix prefix "
                         "groups (nxt_paged_attention_prefix_ex); off = plain decode kernels")
    ap.add_argument("--shard-of", type=int, default=0, metavar="P",
                    help="1 GPU, c2/c5: run rank 0's shard of the P-GPU workload alone, with no "
                         "gather (the per-GPU work of a P-GPU run without its exchange)")
    ap.add_argument("--seed", type=int, default=None,
                    help="another seed for the lengths, tables and values of the workload "
                         "(default: the configuration's own)")
    ap.add_argument("--seqs", type=int, default=0,
                    help="sequences per GPU for c2/c4/c5 (default: the BASELINE size); smaller "
                         "values make the small cases the ncu captures run on")
    return ap.parse_args()


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def build_id():
    """Identity of the loaded kernel build (sources + flags), written by the
    library's Makefile next to the libraries; None when absent."""
    try:
        with open(os.path.join(ROOT, "xllms_b200", "_lib", "build_id")) as f:
            return f.read().strip() or None
    except OSError:
        return None


def ncu_traffic(workload_name: str, alg_bytes: int):
    """DRAM read + write bytes per launch of the attention kernel from the ncu
    capture recorded in profiles/traffic.json, when it was taken on this exact
    workload (same algorithmic bytes) with this exact build (same build id);
    else None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            rec = json.load(f).get(workload_name)
    except Exception:
        return None
    if not rec or int(rec["algorithmic_bytes_per_launch"]) != int(alg_bytes):
        return None
    bid = build_id()
    if bid is None or rec.get("build_id") != bid:
        return None
    return int(rec["dram_read_bytes_per_launch"]) + int(rec["dram_write_bytes_per_launch"])


def make_batch(workload: str, world: int, rank: int, seqs: int = 0, seed=None):
    from xllms_b200 import workloads as W
    kw = {} if seed is None else {"seed": seed}
    if workload == "c2":
        return W.config2(num_seqs=(seqs or 64) * world, world_size=world, rank=rank, **kw)
    if workload == "c5":
        return W.config5(world_size=world, rank=rank, num_seqs=seqs or 512, **kw)
    if world > 1:
        raise SystemExit(f"workload {workload} runs on one GPU")
    if workload == "c4":
        return W.config4(num_seqs=seqs or 256, **kw)
    if workload == "c3":
        return W.config3(**kw)
    return W.CONFIGS[workload](**kw)


# ── clocks during the timed region ────────────────────────────────────────
_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x2: "applications_clocks_setting", 0x10: "sync_boost"}


class ClockSampler:
    """SM clock and clock-event reasons of the job's GPUs, sampled every 10 ms
    by one external `nvidia-smi` process that rank 0 starts before warm-up (no
    sampling work inside the ranks that enqueue GPU work). window() returns a
    handle; summary(handle) keeps the samples whose timestamps fall inside
    that window."""

    FIELDS = "timestamp,pci.bus_id,clocks.sm,clocks.max.sm,clocks_event_reasons.active"

    def __init__(self, torch_devices, enabled: bool = True, period_ms: int = 10):
        import subprocess
        import tempfile
        import torch
        self.enabled = enabled
        self.proc = None
        self.err = None
        if not enabled:
            return
        self.buses = set()
        for d in torch_devices:
            p = torch.cuda.get_device_properties(d)
            self.buses.add(f"{p.pci_bus_id:02x}:{p.pci_device_id:02x}".lower())
        self.tmp = tempfile.NamedTemporaryFile(prefix="clocks_", suffix=".csv", delete=False)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               f"-lms={period_ms}"]
        # Query only the sampled GPUs: a query over every GPU of a large box
        # takes longer than a short timed region.
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id",
                                  "--format=csv,noheader"], capture_output=True, text=True,
                                 timeout=30).stdout
            idx = [ln.split(",")[0].strip() for ln in out.splitlines()
                   if any(b in ln.lower() for b in self.buses)]
            if idx:
                cmd.append("--id=" + ",".join(idx))
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(cmd, stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception as exc:  # pragma: no cover - depends on the box
            self.err = f"nvidia-smi unavailable: {exc}"

    def wait_ready(self, timeout_s: float = 5.0):
        """Blocks until nvidia-smi has written its first sample (it takes a
        few hundred ms to start), so that short timed regions get samples."""
        if self.proc is None:
            return
        t_end = time.time() + timeout_s
        while time.time() < t_end:
            try:
                if os.path.getsize(self.tmp.name) > 0:
                    return
            except OSError:
                return
            time.sleep(0.02)

    @staticmethod
    def now():
        import datetime as _dt
        return _dt.datetime.now()

    def close(self):
        if self.proc is not None:
            time.sleep(0.03)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.proc = None

    def summary(self, t0, t1):
        """Samples of the job's GPUs taken between host times t0 and t1."""
        import datetime as _dt
        if not self.enabled:
            return None
        mhz, maxes, reasons = [], [], 0
        try:
            with open(self.tmp.name) as f:
                lines = f.readlines()
        except OSError as exc:
            lines, self.err = [], str(exc)
        for line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 5:
                continue
            try:
                ts = _dt.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                continue
            if not (t0 <= ts <= t1):
                continue
            bus = parts[1].lower()
            if not any(b in bus for b in self.buses):
                continue
            try:
                mhz.append(float(parts[2]))
                maxes.append(float(parts[3]))
                reasons |= int(parts[4], 16)
            except ValueError:
                continue
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": self.err or "no sample fell inside the timed region"}
        names = sorted({n for bit, n in _REASONS.items() if reasons & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "reasons": names,
                "samples": len(mhz), "gpus": len(self.buses)}


# ── CPU baseline: the reference's own CPU attention on the host cores ─────
def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# The reference CPU attention (examples/run_gpt2.c:63) forms a page's offset
# as the int product page_idx * (page_size * num_heads * head_dim), so its
# pool must stay below 2^31 elements; the sample also bounds the fp32 copy
# of each pool it is given (num_heads wide) to REF_SAMPLE_ELEMS elements.
REF_SAMPLE_ELEMS = 1 << 28


def sample_plan(batch, nseq):
    """(sequences, context lengths) of the CPU sample: the first sequences, up
    to `nseq`, whose pages fit the reference's pool limit; when the first
    sequence alone does not fit, its first tokens that do."""
    bs = batch.block_size
    cap = max(1, min(2**31 - 1, REF_SAMPLE_ELEMS) // (bs * batch.num_heads * batch.head_size))
    seqs, lens, pages = [], [], 0
    for b in range(min(nseq, batch.num_seqs)):
        L = int(batch.seq_lens[b])
        npg = -(-L // bs)
        if pages + npg > cap:
            if not seqs:
                seqs.append(b)
                lens.append(cap * bs)
            break
        seqs.append(b)
        lens.append(L)
        pages += npg
    return seqs, lens


def sample_arrays(batch, nseq, q_t=None, k_t=None, v_t=None):
    """Host arrays (q, k, v, block_tables, seq_lens) of the sample_plan
    sequences with their pages renumbered compactly: copied from the device
    pools when given, else drawn on the host (numpy PCG64, the batch's seed)."""
    import numpy as np
    seqs, lens = sample_plan(batch, nseq)
    if q_t is not None:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from _helpers import gather_subset
        q, k, v, bt, sl = gather_subset(batch, seqs, q_t, k_t, v_t)
        if int(sl[0]) > lens[0]:  # one truncated sequence: keep its first pages
            npg = -(-lens[0] // batch.block_size)
            k, v, bt = k[:npg], v[:npg], np.ascontiguousarray(bt[:, :npg])
            sl = np.array(lens, dtype=np.int32)
        return q, k, v, bt, sl
    from xllms_b200 import workloads as W
    sub = W.make_batch(batch.name + "_sample", np.array(lens), batch.num_heads,
                       batch.num_kv_heads, batch.head_size, batch.dtype, batch.seed,
                       block_size=batch.block_size, slack=0.0, value_std=batch.value_std)
    q, k, v = sub.values_numpy()
    return q, k, v, sub.block_tables, sub.seq_lens


def _kv_label(fmt: str) -> str:
    return "int8" if fmt == "int8" else f"fp8 {fmt}"


def cpu_leg(batch, arrays, seconds: float = 0.0, passes: int = 0, warmup: int = 1):
    """Times the reference CPU path (oracle/_ref, else the oracle port) over the
    sample `arrays` on all host cores. Returns (GB/s, seconds per pass, info)."""
    import numpy as np
    from oracle import oracle as O
    q, k, v, bt, sl = arrays
    if batch.kv_elem_size == 1:  # one-byte pools: the CPU path reads the dequantised values
        fmt = {"e4m3": O.FP8_E4M3, "e5m2": O.FP8_E5M2, "int8": O.KV_INT8}[batch.notes["kv_format"]]
        k = O.fp8_decode(k, fmt) * np.float32(batch.notes["k_scale"])
        v = O.fp8_decode(v, fmt) * np.float32(batch.notes["v_scale"])
    nseq = len(sl)
    cores = host_cores()
    sub_bytes = int(sl.astype(np.int64).sum()) * batch.num_kv_heads * \
        batch.head_size * 2 * batch.kv_es
    sub_bytes += 2 * nseq * batch.num_heads * batch.head_size * batch.elem_size
    sub_bytes += int(((sl.astype(np.int64) + 15) // 16).sum()) * 4 + 4 * nseq
    if O.ref_available():
        kind = "reference"
        kr, vr = O.to_run_gpt2_layout(k, v, batch.num_kv_heads, batch.num_heads,
                                      batch.block_size)
        pt = O.per_token_tables(bt, sl, batch.block_size)
        qf = q.astype(np.float32)

        def one():
            O.reference_attention(qf, kr, vr, pt, sl, batch.block_size, threads=cores)
        what = ("xLLMs examples/run_gpt2.c paged_attention (fp32, GQA via repeated KV heads), "
                "OpenMP over sequences")
    else:
        kind = "port"

        def one():
            O.attention(q, k, v, bt, sl, batch.num_kv_heads, batch.scale, threads=cores)
        what = "oracle/pa_oracle.c restatement, OpenMP over (seq, head)"
    for _ in range(max(1, warmup)):
        one()
    times = []
    t_end = time.perf_counter() + seconds
    while (passes and len(times) < passes) or (not passes and
                                                 (not times or time.perf_counter() < t_end)):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    per = statistics.mean(times)
    cut = int(sl[0]) < int(batch.seq_lens[0])
    info = {"kind": kind, "cores": cores,
            "sample": f"first {nseq} of {batch.num_seqs} sequences "
                      + (f"(sequence 0 cut to its first {int(sl[0])} tokens: the reference "
                         "forms page offsets in 32-bit int) " if cut else "")
                      + f"({int(sl.sum())} context tokens, {sub_bytes / 1e6:.1f} MB algorithmic); "
                      f"{what}; {len(times)} timed passes"}
    return sub_bytes / per / 1e9, per, info


# ── output check (outside the timed regions) ──────────────────────────────
PARITY_RTOL = 1e-3  # north_star: 1e-3 relative error, fp32 accumulation
_PARITY_OK = True    # set by the output check; a failed check makes the exit status 1
_MC_ACTIVE = False   # --gather fused-mc found multicast support


def parity_sample(num_seqs: int):
    """Sequences the output check compares with the oracle: first, last and
    two in between."""
    return sorted({0, num_seqs // 3, (2 * num_seqs) // 3, num_seqs - 1})


def verify_output(batch, q, k, v, full, rank, world, dev, kv_fmt=None, k_scale=1.0,
                  v_scale=1.0):
    """Checks the step's output `full` [B, Hq_total, D] (this rank's gathered
    buffer; the plain output at N = 1). Rank r compares its own heads of the
    parity_sample sequences with the fp64 CPU oracle over its own pools, and
    (N > 1) every rank's buffer must equal this one bit for bit, so together
    every head of every buffer is covered. Returns (ok, worst) reduced over
    the ranks; worst = max |x - ref| / (rtol * max(|ref|, eps))."""
    import numpy as np
    import torch
    from oracle import oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from _helpers import gather_subset
    seqs = parity_sample(batch.num_seqs)
    qs, ks, vs, bt, sl = gather_subset(batch, seqs, q, k, v)
    if kv_fmt:
        fmt = {"e4m3": O.FP8_E4M3, "e5m2": O.FP8_E5M2, "int8": O.KV_INT8}[kv_fmt]
        ref = O.attention_fp8(qs, ks, vs, fmt, k_scale, v_scale, bt, sl, batch.num_kv_heads,
                              batch.scale, block_size=batch.block_size, f64=True)
    else:
        ref = O.attention(qs, ks, vs, bt, sl, batch.num_kv_heads, batch.scale,
                          block_size=batch.block_size, f64=True, threads=host_cores())
    h0 = rank * batch.num_heads
    got = full[seqs][:, h0:h0 + batch.num_heads].float().cpu().numpy()
    ok, worst = O.rel_err_ok(got, ref, PARITY_RTOL)
    ok = bool(ok) and bool(np.isfinite(got).all())
    if world > 1:
        import torch.distributed as dist
        # bit patterns, widened to int32 (every backend gathers int32)
        mine = full.contiguous().view(torch.int16).reshape(-1).to(torch.int32)
        every = torch.empty(world * mine.numel(), dtype=mine.dtype, device=dev)
        dist.all_gather_into_tensor(every, mine)
        ok = ok and bool((every.view(world, -1) == mine.unsqueeze(0)).all())
        t = torch.tensor([0.0 if ok else 1.0, float(worst)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok, worst = t[0].item() == 0.0, t[1].item()
    return ok, float(worst)


# ── our implementation ─────────────────────────────────────────────────────
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from xllms_b200 import _native
    from xllms_b200 import operator_api as PA
    from xllms_b200 import sharding

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.shard_of > 1:
        if world > 1 or args.workload not in ("c2", "c5"):
            raise SystemExit("--shard-of runs one shard of c2 / c5 on one GPU")
        batch = make_batch(args.workload, args.shard_of, 0, args.seqs, args.seed)
    else:
        batch = make_batch(args.workload, world, rank, args.seqs, args.seed)
    fp8 = args.kv != "fp16"
    if fp8 and (world > 1 or args.workload in ("c1", "c4")):
        raise SystemExit("--kv e4m3 / e5m2 / int8 runs configs 2, 3 and 5 on one GPU")
    if fp8:
        q, k, v, k_scale, v_scale = batch.values_torch_fp8(dev, args.kv)
    else:
        q, k, v = batch.values_torch(dev)
    bt, sl = batch.tables_torch(dev)
    out = torch.empty_like(q)
    gathered = full = fg = None
    fused = world > 1 and args.gather in ("fused", "fused-mc")
    if fused:
        want_mc = args.gather == "fused-mc"
        if want_mc:
            # every rank must take the same path: agree on multicast support first
            ok = torch.tensor([1 if sharding.multicast_supported(dev) else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            want_mc = bool(ok.item())
        fg = sharding.FusedHeadGather(batch.num_seqs, batch.total_heads, batch.head_size,
                                      batch.dtype_size, world, rank, sharding.torch_exchange(),
                                      dev, multicast=want_mc)
        global _MC_ACTIVE
        _MC_ACTIVE = fg.multicast
    elif world > 1:
        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev)
        full = torch.empty((batch.num_seqs, batch.total_heads, batch.head_size),
                           dtype=out.dtype, device=dev)
    lib = _native.xpa()
    path = PA.kernel_path(k, v, batch.num_heads, batch.head_size, batch.num_kv_heads,
                          batch.block_size, batch.dtype_size, batch.kv_block_stride,
                          batch.kv_head_stride)
    split = PA.workspace_size(batch.num_seqs, batch.num_heads, batch.head_size,
                              batch.num_kv_heads, batch.max_blocks, batch.block_size,
                              batch.dtype_size) > 0
    cascade = (args.prefix == "on" and bool(batch.prefix_groups) and world == 1
               and path == _native.NXT_PA_PATH_TMA_MMA)
    groups = PA.PrefixGroups(batch.prefix_groups, batch.num_seqs, dev) if cascade else None
    # attention kernel (+ split-context merge) (+ the fused gather's barrier);
    # cascade: prefix kernel + suffix kernel + merge
    launches_per_step = (3 if cascade else
                         1 + (1 if split else 0) + (1 if fused else 0))

    def step():
        if fused:
            fg.run(q, k, v, bt, sl, batch.scale, batch.num_blocks)
            return
        if cascade:
            PA.paged_attention_prefix(q, k, v, bt, sl, groups, out=out,
                                      num_blocks=batch.num_blocks)
            return
        if fp8:
            PA.paged_attention_fp8(q, k, v, bt, sl, args.kv, k_scale, v_scale, out=out,
                                   num_blocks=batch.num_blocks)
            return
        PA.paged_attention(q, k, v, bt, sl, out=out, num_blocks=batch.num_blocks)
        if world > 1:
            sharding.gather_heads(out, gathered)
            sharding.interleave_heads(gathered, full)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # rank 0 samples its own GPU; every rank runs the same work in lockstep
    sampler = ClockSampler([local_rank], enabled=(rank == 0))
    sampler.wait_ready()
    for _ in range(args.warmup):
        step()
    barrier()
    st = PA.device_status(clear=True)
    if st:
        raise SystemExit(f"device status after warm-up: {st:#x}")

    K = args.steps
    # Timed region 1: K plain steps -> value, ms_per_step, clocks. With
    # --graph the step is captured once and replayed K times (same kernels,
    # no host launch work between them).
    graph = None
    if args.graph:
        if world > 1:
            raise SystemExit("--graph is a 1-GPU option")
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()  # a call on the capture stream before capturing
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        # capture on the stream that already holds the library's workspace
        # (allocating one would not be allowed while capturing)
        with torch.cuda.graph(graph, stream=side):
            step()
        graph.replay()
        torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    c0 = ClockSampler.now()
    torch.cuda.nvtx.range_push("timed steps")
    start.record()
    for _ in range(K):
        if graph is not None:
            graph.replay()
        else:
            step()
    stop.record()
    torch.cuda.nvtx.range_pop()
    barrier()
    c1 = ClockSampler.now()
    t_step = start.elapsed_time(stop) / K
    # output of the device-resident run, checked against the oracle
    resident = (fg.output(fg.step) if fused else (full if world > 1 else out)).clone()
    parity = verify_output(batch, q, k, v, resident, rank, world, dev,
                           kv_fmt=args.kv if fp8 else None,
                           k_scale=k_scale if fp8 else 1.0, v_scale=v_scale if fp8 else 1.0)

    # Timed region 2: K steps with events recorded by the library right around
    # the attention kernel -> its own mean duration for the roofline. (Kept
    # out of region 1: an event between the attention kernel and the merge
    # kernel stops the merge's programmatic launch from overlapping the tail.)
    # The library records ev_a / ev_b around the attention kernel and ev_c
    # after the merge; ev_d closes the step (after the fused gather's barrier,
    # or the NCCL gather), which gives the per-rank split of a step.
    ev_a, ev_b, ev_c, ev_d = ([torch.cuda.Event(enable_timing=True) for _ in range(K)]
                              for _ in range(4))
    for e in ev_a + ev_b + ev_c + ev_d:
        e.record()  # materialise the CUDA event handles
    barrier()
    torch.cuda.nvtx.range_push("profiled steps")
    for i in range(K):
        lib.nxt_paged_attention_profile_next_ex(ev_a[i].cuda_event, ev_b[i].cuda_event,
                                                ev_c[i].cuda_event)
        step()
        ev_d[i].record()
    torch.cuda.nvtx.range_pop()
    barrier()
    t_kern = statistics.mean(a.elapsed_time(b) for a, b in zip(ev_a, ev_b))
    split = [statistics.mean(a.elapsed_time(b) for a, b in zip(x, y))
             for x, y in ((ev_a, ev_b), (ev_b, ev_c), (ev_c, ev_d))]
    st = PA.device_status(clear=True)
    if st:
        raise SystemExit(f"device status after timing: {st:#x}")

    # ── e2e through the backend plugin (C ABI) with host buffers ───────────
    if args.no_e2e:
        if fg is not None:
            fg.close(dist.barrier)
        sampler.close()
        return _finish(args, rank, world, batch, path, launches_per_step, t_step, t_kern, None,
                       sampler.summary(c0, c1), None, q, k, v, 0, 0, dev, cascade,
                       parity=parity, split=split)
    plugin = PA.CudaBackendPlugin()
    # One pinned staging buffer holds the step's inputs (Q | block tables |
    # seq_lens), so each step issues a single host->device copy; the device
    # side is one buffer viewed as the three tensors.
    # A cascade step's prefix groups (prefix pages per sequence, group
    # offsets, members) ride in the same copy.
    host_parts = [q.cpu(), bt.cpu(), sl.cpu()]
    if cascade:
        host_parts += [torch.from_numpy(a) for a in
                       PA.PrefixGroups.host_arrays(batch.prefix_groups, batch.num_seqs)]
    sizes = [t.numel() * t.element_size() for t in host_parts]

    def make_io():
        """Pinned host staging + its device copy (viewed as the step's input
        tensors), a device output and a pinned host output."""
        io = {"stage_h": torch.empty(sum(sizes), dtype=torch.uint8).pin_memory()}
        io["stage_d"] = torch.empty_like(io["stage_h"], device=dev)
        views, o = [], 0
        for t, n in zip(host_parts, sizes):
            io["stage_h"][o:o + n].copy_(t.reshape(-1).view(torch.uint8))
            views.append(io["stage_d"][o:o + n].view(t.dtype).view(t.shape))
            o += n
        io["q"], io["bt"], io["sl"] = views[:3]
        io["groups"] = (PA.PrefixGroups(batch.prefix_groups, batch.num_seqs,
                                        prefix_pages=views[3], offsets=views[4],
                                        members=views[5]) if cascade else None)
        io["out_d"] = torch.empty_like(out)
        io["out_h"] = torch.empty((batch.num_seqs, batch.total_heads, batch.head_size),
                                  dtype=out.dtype).pin_memory()
        io["pa_in"] = None if fp8 else PA.make_input(io["q"], k, v, io["bt"], io["sl"],
                                                     scale=batch.scale,
                                                     stream=torch.cuda.current_stream())
        return io

    io0 = make_io()
    stage_h, out_h = io0["stage_h"], io0["out_h"]

    def compute(io):
        """One step through the C ABI on the current stream; returns the
        device tensor that holds its [B, Hq_total, D] result."""
        if fused:
            # the C-ABI sharded entry point (the plugin descriptor has no shard fields)
            return fg.run(io["q"], k, v, io["bt"], io["sl"], batch.scale, batch.num_blocks)
        if cascade:
            # the C-ABI cascade entry point (the plugin descriptor has no group fields)
            PA.paged_attention_prefix(io["q"], k, v, io["bt"], io["sl"], io["groups"],
                                      out=io["out_d"], num_blocks=batch.num_blocks)
        elif fp8:
            # the C-ABI fp8 entry point (the plugin descriptor has no KV format)
            PA.paged_attention_fp8(io["q"], k, v, io["bt"], io["sl"], args.kv, k_scale, v_scale,
                                   out=io["out_d"], num_blocks=batch.num_blocks)
        elif plugin.run(io["pa_in"], io["out_d"]) != 0:
            raise SystemExit("nxt_backend_run failed")
        if world > 1:
            sharding.gather_heads(io["out_d"], gathered)
            sharding.interleave_heads(gathered, full)
            return full
        return io["out_d"]

    def e2e_step():
        io0["stage_d"].copy_(io0["stage_h"], non_blocking=True)
        io0["out_h"].copy_(compute(io0), non_blocking=True)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0 = ClockSampler.now()
    torch.cuda.nvtx.range_push("e2e steps")
    e_start.record()
    for _ in range(K):
        e2e_step()
    e_stop.record()
    torch.cuda.nvtx.range_pop()
    barrier()
    e1 = ClockSampler.now()
    # The same steps with the host waiting for each step's output before it
    # enqueues the next, as a decode loop must (the idle gaps are timed too).
    h_start, h_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("e2e host-synced steps")
    h_start.record()
    for _ in range(K):
        e2e_step()
        torch.cuda.current_stream().synchronize()
    h_stop.record()
    torch.cuda.nvtx.range_pop()
    barrier()
    # Pipelined (1 GPU): two input / output sets; a step's host->device copy
    # runs on its own stream during the previous step's compute and its
    # device->host read during the next step's, as a serving loop overlaps
    # them. Every copy of every step is still inside the timed region.
    t_e2e_pipe = None
    if world == 1:
        ios = [io0, make_io()]
        comp, up, down = torch.cuda.current_stream(), torch.cuda.Stream(), torch.cuda.Stream()
        up_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        down_done = [torch.cuda.Event() for _ in range(2)]

        def piped(n, t_start=None, t_stop=None):
            if t_start is not None:
                t_start.record(comp)
            up.wait_stream(comp)
            down.wait_stream(comp)
            for i in range(n):
                b, io = i & 1, ios[i & 1]
                with torch.cuda.stream(up):
                    if i >= 2:
                        up.wait_event(comp_done[b])  # set b's inputs consumed
                    io["stage_d"].copy_(io["stage_h"], non_blocking=True)
                    up_done[b].record(up)
                comp.wait_event(up_done[b])
                if i >= 2:
                    comp.wait_event(down_done[b])  # set b's output read back
                res_d = compute(io)
                comp_done[b].record(comp)
                with torch.cuda.stream(down):
                    down.wait_event(comp_done[b])
                    io["out_h"].copy_(res_d, non_blocking=True)
                    down_done[b].record(down)
            comp.wait_stream(down)
            if t_stop is not None:
                t_stop.record(comp)

        piped(max(3, args.warmup))
        barrier()
        p_start = torch.cuda.Event(enable_timing=True)
        p_stop = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("e2e pipelined steps")
        piped(K, p_start, p_stop)
        torch.cuda.nvtx.range_pop()
        barrier()
        t_e2e_pipe = p_start.elapsed_time(p_stop) / K
        for io in ios:
            if not torch.equal(io["out_h"].to(dev), resident):
                raise SystemExit("pipelined e2e output differs from the device-resident run")
    sampler.close()
    clocks, clocks_e2e = sampler.summary(c0, c1), sampler.summary(e0, e1)
    t_e2e = e_start.elapsed_time(e_stop) / K
    t_e2e_sync = h_start.elapsed_time(h_stop) / K
    if not torch.equal(out_h.to(dev), resident):
        raise SystemExit("e2e output differs from the device-resident run")
    plugin.close()
    if fg is not None:
        fg.close(dist.barrier)
    h2d = stage_h.numel()
    d2h = out_h.numel() * out_h.element_size()
    return _finish(args, rank, world, batch, path, launches_per_step, t_step, t_kern, t_e2e,
                   clocks, clocks_e2e, q, k, v, h2d, d2h, dev, cascade, parity=parity,
                   split=split, t_e2e_sync=t_e2e_sync, t_e2e_pipe=t_e2e_pipe)


def _finish(args, rank, world, batch, path, launches_per_step, t_step, t_kern, t_e2e, clocks,
            clocks_e2e, q, k, v, h2d, d2h, dev, cascade=False, parity=(True, 0.0), split=None,
            t_e2e_sync=None, t_e2e_pipe=None):
    import torch
    import torch.distributed as dist
    K = args.steps
    bytes_rank = batch.algorithmic_bytes()
    ub_rank = batch.algorithmic_bytes(unique=True) if args.workload == "c4" else bytes_rank
    kv_rank = batch.kv_bytes()
    global _PARITY_OK
    _PARITY_OK = bool(parity[0])
    split = split or [0.0, 0.0, 0.0]
    per_rank = [split]
    if world > 1:
        t = torch.tensor([t_step, t_kern, t_e2e or 0.0, t_e2e_sync or 0.0], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_step, t_kern, t_e2e, t_e2e_sync = (float(x) for x in t.tolist())
        t_e2e = t_e2e or None
        t_e2e_sync = t_e2e_sync or None
        mine = torch.tensor(split, dtype=torch.float64, device=dev)
        every = torch.empty(world * 3, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(every, mine)
        per_rank = every.view(world, 3).tolist()
        s = torch.tensor([bytes_rank, ub_rank, kv_rank, h2d, d2h], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        tot_bytes, tot_ub, tot_kv, h2d, d2h = (float(x) for x in s.tolist())
    else:
        tot_bytes, tot_ub, tot_kv = float(bytes_rank), float(ub_rank), float(kv_rank)
    t_e2e_best = min(x for x in (t_e2e, t_e2e_pipe) if x) if t_e2e else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, per, info = cpu_leg(batch, sample_arrays(batch, 8, q, k, v), args.cpu_seconds)
        cpu = dict(value=round(gbs, 3), unit="GB/s", **info)

    if rank != 0:
        return None
    peak, peak_src = hbm_peak()
    value = tot_bytes / (t_step * 1e-3) / 1e9
    kern_gbs = ub_rank / (t_kern * 1e-3) / 1e9  # per GPU: the kernel's own bytes per launch
    seqs_total = batch.num_seqs  # every rank decodes every sequence for its heads
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(t_step, 5),
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "c5" else "weak",
        "vs_baseline": None,
        "dtype": "f16" if batch.kv_elem_size != 1 else
                 f"f16 (Q, out), {_kv_label(batch.notes['kv_format'])} KV",
        "data": "synthetic: seeded block tables/lengths (numpy PCG64); Q/K/V N(0,1)*std "
                "drawn on the device (torch CUDA generator)" +
                (f"; K/V quantised to {_kv_label(batch.notes['kv_format'])} with one scale "
                 "per pool" if batch.kv_elem_size == 1
                 else ""),
        "config": {
            "workload": batch.name,
            "num_seqs": batch.num_seqs,
            "num_heads": batch.total_heads,
            "num_kv_heads": batch.num_kv_heads * world,
            "kv_heads_per_gpu": batch.num_kv_heads,
            "head_size": batch.head_size,
            "block_size": batch.block_size,
            "max_blocks_per_seq": batch.max_blocks,
            "context_tokens": batch.context_tokens(),
            "parallelism": "single GPU" if world == 1 else
                           (f"KV-head sharding x{world}, output gather fused into the kernels "
                            "(NVLink peer stores + bounded cross-GPU barrier)"
                            if args.gather == "fused" else
                            f"KV-head sharding x{world}, output gather fused into the kernels "
                            "(one multimem store per 16-byte chunk through NVSwitch multicast "
                            "+ bounded cross-GPU barrier)"
                            if args.gather == "fused-mc" and _MC_ACTIVE else
                            f"KV-head sharding x{world}, output gather fused into the kernels "
                            "(peer stores into symmetric-memory buffers; no multicast support) "
                            "+ bounded cross-GPU barrier" if args.gather == "fused-mc" else
                            f"KV-head sharding x{world} + NCCL all-gather of outputs"),
            "l2": f"no flush: each step reads {tot_kv / world / 1e9:.2f} GB of KV per GPU "
                  f"(> {L2_BYTES >> 20} MB L2)",
            "timing": "CUDA graph of one step, K replays" if args.graph else "K enqueued steps",
            "path": {1: "tma_mma", 2: "generic"}.get(path, "none") +
                    (" + shared-prefix (cascade) kernel" if cascade else "") +
                    (f" ({_kv_label(batch.notes['kv_format'])} KV variant)"
                     if batch.kv_elem_size == 1 else ""),
            "kv_cache": batch.notes.get("kv_format", "fp16"),
            **({"shard_of": args.shard_of} if args.shard_of > 1 else {}),
            **({"seed": args.seed} if args.seed is not None else {}),
        },
        "pct_hbm_peak": round(100.0 * (tot_ub / world) / (t_step * 1e-3) / 1e9 / peak, 2),
        "seq_tokens_per_s": round(seqs_total / (t_step * 1e-3), 1),
        "context_tokens_per_s": round(batch.context_tokens() / (t_step * 1e-3), 1),
        "kv_gbs": round(tot_kv / (t_step * 1e-3) / 1e9, 2),
        "roofline": {
            "bound": "hbm",
            "kernel": ("pa_prefix_kernel + pa_tma_mma_kernel (events span both)" if cascade
                       else "pa_tma_mma_kernel" if path == 1 else "pa_generic_kernel"),
            "achieved": round(kern_gbs, 2),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(kern_gbs / peak, 4),
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                           else "fallback 6.65 TB/s",
            "kernel_ms": round(t_kern, 5),
            "traffic": ncu_traffic(batch.name, ub_rank),
            "build_id": build_id(),
            "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "bytes_per_launch": ub_rank,
        },
        "e2e": None if t_e2e is None else {
            "value": round(tot_bytes / (t_e2e_best * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "ms_per_step": round(t_e2e_best, 5),
            "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "timing": ("the faster of two ways to run the steps, every copy of every step inside "
                       "the timed region: " + ("pipelined" if t_e2e_best == t_e2e_pipe else
                                               "enqueued") + " (both below)"),
            "enqueued": {
                "value": round(tot_bytes / (t_e2e * 1e-3) / 1e9, 2),
                "ms_per_step": round(t_e2e, 5),
                "what": "one input / output set, copies and compute in stream order, steps "
                        "enqueued back to back",
            },
            "pipelined": None if t_e2e_pipe is None else {
                "value": round(tot_bytes / (t_e2e_pipe * 1e-3) / 1e9, 2),
                "ms_per_step": round(t_e2e_pipe, 5),
                "what": "two input / output sets; each step's H2D copy runs on its own stream "
                        "during the previous step's compute and its D2H read during the next "
                        "step's (1 GPU)",
            },
            "api": ("nxt_paged_attention_prefix_ex (libxpa.so); per step one pinned H2D copy "
                    "(Q, block tables, seq_lens, prefix groups) and one D2H copy of the output"
                    if cascade else
                    "nxt_paged_attention_fp8_ex (libxpa.so); per step one pinned H2D copy "
                    "(Q, block tables, seq_lens) and one D2H copy of the output"
                    if batch.kv_elem_size == 1 else
                    "nxt_backend_run (libxllm_cuda_backend.so); per step one pinned H2D copy "
                    "(Q, block tables, seq_lens) and one D2H copy of the output"),
            "clocks": clocks_e2e,
            "host_synced": None if t_e2e_sync is None else {
                "value": round(tot_bytes / (t_e2e_sync * 1e-3) / 1e9, 2),
                "ms_per_step": round(t_e2e_sync, 5),
                "what": "the same steps, the host waiting for each step's output before "
                        "enqueueing the next (idle gaps included)",
            },
        },
        "parity_ok": bool(parity[0]),
        "parity_worst": round(float(parity[1]), 4),
        "parity_check": (f"sequences {parity_sample(batch.num_seqs)} of the gathered output vs "
                         f"the fp64 CPU oracle over each rank's pools, |x-ref| <= "
                         f"{PARITY_RTOL:g}*max(|ref|, 0.01*rms(ref)); worst = largest "
                         "|x-ref| / that bound (<= 1 passes)" +
                         ("; every rank's gathered buffer bitwise equal" if world > 1 else "")),
        "per_rank": {
            "attn_ms": [round(x[0], 5) for x in per_rank],
            "merge_ms": [round(x[1], 5) for x in per_rank],
            "barrier_ms": [round(x[2], 5) for x in per_rank],
            "what": "mean per step over K steps with events between the kernels: attention "
                    "kernel; split-context merge; from the merge to the end of the step (the "
                    "fused gather's cross-GPU barrier, or the NCCL all-gather + interleave)",
        },
        "clocks": clocks,
        "gpu_launches": launches_per_step * K * world,
        "gpu_launches_per_rank": launches_per_step * K,
    }
    if args.workload == "c4":
        line["unique_kv_gbs"] = round(tot_ub / (t_step * 1e-3) / 1e9, 2)
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_reference(args, rank, world):
    """The reference's own CPU attention on the host cores, on a sample of this
    arm's workload (sample_plan: up to the first 8 sequences); rank 0 only, one
    sample pass per step."""
    if rank != 0:
        return None
    batch = make_batch(args.workload, world, 0, args.seqs, args.seed)
    arrays = sample_arrays(batch, 8)
    seqs = len(arrays[4])
    gbs, per, info = cpu_leg(batch, arrays, passes=max(1, args.steps), warmup=args.warmup)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic, the ours arm's seeded workload (the sample's sequences, host-drawn "
                "values)",
        "config": {"workload": batch.name, "sample_seqs": seqs, "num_heads": batch.total_heads,
                   "num_kv_heads": batch.num_kv_heads * world, "head_size": batch.head_size,
                   "block_size": batch.block_size},
        "seq_tokens_per_s": round(seqs / per, 2),
        "cpu_baseline": dict(value=round(gbs, 3), unit="GB/s", **info),
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_activation(args):
    """One activation operator on a [tokens, 2 d] fp16 input (Llama-3-8B MLP:
    d = 14336): algorithmic bytes = input + output; roofline HBM."""
    import torch
    from oracle import oracle as O
    from xllms_b200 import _native
    from xllms_b200 import operator_api as PA
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    op = PA.ACTIVATIONS[args.act_op]
    gated = op <= _native.NXT_ACT_GELU_TANH_AND_MUL
    T, d = args.act_tokens, args.act_d
    width = 2 * d if gated else d
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    x = (torch.randn(T, width, generator=g, device=dev) * 2).to(torch.float16)
    out = torch.empty(T, d, dtype=torch.float16, device=dev)
    nbytes = (x.numel() + out.numel()) * 2
    step = lambda: PA.activation(args.act_op, x, out=out)
    sampler = ClockSampler([0])
    sampler.wait_ready()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    K = args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0 = ClockSampler.now()
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    c1 = ClockSampler.now()
    t_step = e0.elapsed_time(e1) / K
    # e2e: the input from pinned host memory, the output back, every step
    x_h = x.cpu().pin_memory()
    out_h = torch.empty(T, d, dtype=torch.float16).pin_memory()
    x_d = torch.empty_like(x)

    def e2e():
        x_d.copy_(x_h, non_blocking=True)
        PA.activation(args.act_op, x_d, out=out)
        out_h.copy_(out, non_blocking=True)
    for _ in range(3):
        e2e()
    torch.cuda.synchronize()
    E = max(1, K // 4)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(E):
        e2e()
    f1.record()
    torch.cuda.synchronize()
    t_e2e = f0.elapsed_time(f1) / E
    sampler.close()
    cpu = None
    if not args.no_cpu_baseline:
        rows = max(1, min(T, 64))
        xs = x[:rows].cpu().numpy()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0) or n == 0:
            O.activation(op, xs)
            n += 1
        dt = (time.perf_counter() - t0) / n
        cpu = {"value": round(rows * (width + d) * 2 / dt / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"{rows} of {T} rows, oracle/act_oracle.c (libm, 1 thread)"}
    peak, peak_src = hbm_peak()
    gbs = nbytes / (t_step * 1e-3) / 1e9
    line = {
        "metric": f"activation {args.act_op} GB/s (% of HBM peak)",
        "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": K, "warmup": args.warmup,
        "ms_per_step": round(t_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: N(0,1)*2 fp16 drawn on the device (torch CUDA generator)",
        "config": {"workload": f"act_{args.act_op}", "tokens": T, "d": d,
                   "input": f"[{T}, {width}] fp16", "output": f"[{T}, {d}] fp16",
                   "l2": f"no flush: {nbytes / 1e6:.0f} MB per step (> {L2_BYTES >> 20} MB L2)"},
        "pct_hbm_peak": round(100.0 * gbs / peak, 2),
        "roofline": {"bound": "hbm", "kernel": "act_vec_kernel", "achieved": round(gbs, 2),
                     "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                     "bytes_per_launch": nbytes, "traffic": None},
        "e2e": {"value": round(nbytes / (t_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(t_e2e, 5), "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 2,
                "api": "nxt_activation_ex (libxpa.so), pinned host buffers"},
        "clocks": sampler.summary(c0, c1),
        "gpu_launches": K,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def main():
    args = parse_args()
    if args.workload == "act":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the activation workload has no reference CPU arm"}), flush=True)
            return
        print(json.dumps(run_activation(args)), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if args.gpus != 1 or world != 1:
            print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    if not _PARITY_OK:
        print(f"rank {rank}: output check against the oracle failed", file=sys.stderr)
        sys.exit(1)


if __name__ == "__main__":
    main()
