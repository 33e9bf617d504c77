"""Benchmark of torch_kunlun's int16-quantised dense-op path on B200.

Headline, at every GPU count (N = 1 included): the tensor-parallel
SiLU-gated MLP (the multi-GPU workload) -- x fp16 [16384, 8192] ~N(0,1),
gate/up weights [28672, 8192] split by output rows (column-parallel), down
weight [8192, 28672] split by input columns (row-parallel), all ~N(0,0.02);
h = T(silu(x Wg^T)) * (x Wu^T), y = sum over ranks of h_r Wd_r^T, the partial
sums reduce-scattered by rows: by default over peer memory (each finished
row block of the down projection copied by copy engines into its owner's
buffer over NVLink while the next block computes, then summed in rank order
in fp32 with one rounding), with the `bkcl` (NCCL) reduce-scatter and
all-reduce measured beside it.
Every linear is the int16-quantised GEMM; each rank quantises its own shards.
A step is one forward of the whole MLP over the 16384 tokens.  Metric:
aggregate int16 TOPS = 3 * 2 * 16384 * 8192 * 28672 / step time (strong
scaling: the total work is fixed, split over N ranks).

Outside the timed region every rank checks parity (`parity` / `parity_ok`):
its GEMMs bit-exact against the oracle on sampled rows of its own shards,
the SiLU gate within its stated bound, and its reduced rows against the
rank-ordered fp32 sum of every rank's partial (bit-exact for the
deterministic reductions, within the fp16 summation bound for NCCL's).

On the N = 1 line (skipped with --no-extra) the other configs are objects,
each with its own roofline: the single linear 2048x4096x4096 (cfg1, with its
own end-to-end number), the 4096^3 linear, the BERT-base encoder block
(tokens/s and per-op shares), the attention-score bmm chain, the ResNet-50
convolutions and the HBM-bound row kernels.

Arms:
  default            the kunlun device (hand-written sm_100a kernels)
  --impl reference   the reference path on the host cores: the oracle's CPU
                     restatement (oracle/), rank 0 only
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# ---- the tensor-parallel MLP --------------------------------------------------

TP_T, TP_H, TP_F = 16384, 8192, 28672
TP_OPS = 3 * 2 * TP_T * TP_H * TP_F
TP_BLOCK = 512  # weights are drawn in blocks of 512 rows/columns, so shards agree for every N
METRIC = "int16-quant TP-MLP effective TOPS (aggregate over GPUs)"
WORKLOAD = ("tensor-parallel SiLU-gated MLP: x[16384,8192] fp16, gate/up [28672,8192] column-parallel, "
            "down [8192,28672] row-parallel, partial sums reduced over bkcl (NCCL)")
REF_ROWS = 16  # tokens per reference-arm / cpu_baseline sample

# ---- the single-GPU configs (objects on the N = 1 line) ------------------------

M1, N1, K1 = 2048, 4096, 4096
BERT_B, BERT_L, BERT_H, BERT_HEADS, BERT_F, BERT_TAIL = 32, 512, 768, 12, 3072, 64
BERT_WORKLOAD = ("BERT-base encoder block forward: hidden 768, 12 heads x 64, FFN 3072 gelu, "
                 "post-LN eps 1e-12, batch 32 x seq 512 fp16, additive mask on the last 64 keys")
BMM_B, BMM_M, BMM_E = 64, 512, 128
BMM_OPS = 2 * (2 * BMM_B * BMM_M * BMM_M * BMM_E)
CONV_CASES = [  # (name, C, F, H, k, pad, groups, bias)
    ("1x1 256->64 @56", 256, 64, 56, 1, 0, 1, False),
    ("3x3 64->64 @56 pad1", 64, 64, 56, 3, 1, 1, False),
    ("3x3 256->256 @14 pad1 +bias", 256, 256, 14, 3, 1, 1, True),
    ("3x3 depthwise g=512 @7 pad1", 512, 512, 7, 3, 1, 512, False),
]
CONV_N = 64

PROFILES = os.path.join(ROOT, "profiles")


# ---- peaks and roofline objects ------------------------------------------------

def load_peaks():
    """Roofline denominators.  HBM: the driver's measured copy bandwidth.
    int16 GEMM: the int8 dense rate (twice the measured bf16 dense rate on
    B200) divided by the 4 limb MMAs of one int16 MAC, from the burst figure
    for kernels timed alone and the sustained one for long steps."""
    d, src = {}, "fallback figures of this pool (MEASURED_PEAKS.json absent)"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        src = "MEASURED_PEAKS.json (driver-measured)"
    except (OSError, ValueError):
        pass
    bf16 = float(d.get("bf16_tflops") or 1590.0)
    bf16_s = float(d.get("bf16_tflops_sustained") or 1400.0)
    return {"hbm_gbs": float(d.get("hbm_gbs") or 6650.0), "bf16_tflops": bf16,
            "bf16_tflops_sustained": bf16_s, "int16_burst": 2.0 * bf16 / 4.0,
            "int16_sustained": 2.0 * bf16_s / 4.0, "source": src}


def roofline(bound, achieved, peak, unit, peak_source, traffic=None, traffic_source=None, **extra):
    r = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
         "frac": achieved / peak if peak else None, "peak_source": peak_source,
         "traffic": traffic}
    if traffic_source:
        r["traffic_source"] = traffic_source
    r.update(extra)
    return r


def ncu_traffic(name):
    """dram bytes per launch recorded in a committed ncu summary, if present."""
    p = os.path.join(PROFILES, name)
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip()), "profiles/" + name + " (committed ncu summary)"
    except OSError:
        pass
    return None, None


def int16_peak_source(peaks, which):
    bf = peaks["bf16_tflops"] if which == "burst" else peaks["bf16_tflops_sustained"]
    return (f"2 x {bf:.1f} TF/s bf16 dense ({which}, {peaks['source']}) as the int8 rate, "
            "/ 4 limb MMAs per int16 MAC")


# ---- timing ------------------------------------------------------------------------

def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, polled through
    NVML every 5 ms while the timed region runs.  The GPU is found by UUID so
    CUDA and NVML device orderings cannot disagree."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.cuda_index).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            return self
        self._stop = threading.Event()

        def poll():
            while not self._stop.is_set():
                try:
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         int(get_reasons(h))))
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "NVML, 5 ms"}


def timed_steps(step, steps, warmup, flush, kunlun):
    """Per-step device time with CUDA events on the launching stream; the L2
    flush between steps is outside the events (and, being ~80 us of device
    work, lets the host enqueue the next step before the GPU reaches it)."""
    for _ in range(warmup):
        step()
        flush()
    kunlun.synchronize()
    times = []
    for _ in range(steps):
        e0 = kunlun.Event(enable_timing=True)
        e1 = kunlun.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        flush()
        times.append((e0, e1))
    kunlun.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def make_flush(dev, kunlun):
    """L2 flush between timed steps: the library's amax kernel reading a
    512 MiB buffer (four times L2) on the launching stream, outside the
    events.  The step that follows finds none of its data in L2, and the
    previous step's dirty lines have been written back during the flush
    rather than inside the next step."""
    import torch
    from torch_kunlun_b200 import ops
    scratch = torch.ones(256 * 1024 * 1024, dtype=torch.float16).to(dev)

    def flush():
        ops.amax(scratch)
    return flush


L2_NOTE = ("flushed between steps: a 512 MiB device read outside the timed events (no data of the step in L2, "
           "no dirty lines left to write back)")


def step_stats(times):
    return {"mean": sum(times) / len(times), "min": min(times), "median": statistics.median(times),
            "max": max(times)}


# ---- the C-ABI GEMM kernel alone --------------------------------------------------

class LimbGemm:
    """One int16 GEMM out[M,N] = q(a) q(w)^T launched alone through the C ABI
    (tk_qgemm_from_limbs) on operands quantised once beforehand: the device
    time of the GEMM kernel itself, for the roofline."""

    def __init__(self, a, w, out):
        import torch
        from torch_kunlun_b200 import _capi as C
        self.C, self.L = C, C.lib()
        self.a, self.w, self.out = a, w, out
        M, K = a.shape
        N = w.shape[0]
        ld = (K + 15) // 16 * 16
        dev = a.device
        self.la = torch.empty(2 * M * ld, dtype=torch.int8, device=dev)
        self.lb = torch.empty(2 * N * ld, dtype=torch.int8, device=dev)
        self.amax = torch.empty(2, dtype=torch.float32, device=dev)
        d = C.QGemmDesc()
        d.dtype = C.TK_DTYPE_F16 if a.dtype == torch.float16 else C.TK_DTYPE_F32
        d.batch, d.m, d.n, d.k = 1, M, N, K
        d.out = out.data_ptr()
        d.out_sb, d.out_sm = M * N, out.stride(0)
        d.alpha, d.beta, d.act, d.per_slice_scales = 1.0, 0.0, 0, 1
        self.d, self.M, self.N, self.K = d, M, N, K

    def prepare(self, kunlun):
        C, L = self.C, self.L
        st = kunlun.current_stream().stream_id
        dt = self.d.dtype
        C.check(L.tk_amax(dt, self.a.data_ptr(), 1, 0, self.M * self.K, self.amax.data_ptr(), st), "amax")
        C.check(L.tk_amax(dt, self.w.data_ptr(), 1, 0, self.N * self.K, self.amax.data_ptr() + 4, st), "amax")
        C.check(L.tk_quantize_limbs(dt, self.a.data_ptr(), 1, self.M, self.K, 0, self.a.stride(0), 1,
                                    self.amax.data_ptr(), 0, self.la.data_ptr(), st), "quantise")
        C.check(L.tk_quantize_limbs(dt, self.w.data_ptr(), 1, self.N, self.K, 0, self.w.stride(0), 1,
                                    self.amax.data_ptr() + 4, 0, self.lb.data_ptr(), st), "quantise")

    def launch(self, kunlun):
        st = kunlun.current_stream().stream_id
        self.C.check(self.L.tk_qgemm_from_limbs(ctypes.byref(self.d), self.la.data_ptr(), self.lb.data_ptr(),
                                                self.amax.data_ptr(), self.amax.data_ptr() + 4, st),
                     "tk_qgemm_from_limbs")

    def ms(self, kunlun, flush, iters=10, warmup=3):
        self.prepare(kunlun)
        ts = timed_steps(lambda: self.launch(kunlun), iters, warmup, flush, kunlun)
        return sum(ts) / len(ts)

    def ops(self):
        return 2 * self.M * self.N * self.K


# ---- tensor-parallel MLP: data -------------------------------------------------------

def _block(shape, seed, scale):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).half()


def tp_inputs(rank, world, dev):
    """x [T, H] and this rank's shards.  Every weight is drawn in blocks of
    512 rows (gate, up) or columns (down) with one seed per block, so rank r
    of N ranks holds exactly rows/columns [r F/N, (r+1) F/N) of the same
    full weights for every N."""
    import torch
    fr = TP_F // world
    b0, nb = rank * fr // TP_BLOCK, fr // TP_BLOCK
    x = torch.empty(TP_T, TP_H, dtype=torch.float16, device=dev)
    for b in range(TP_T // 2048):
        x[b * 2048:(b + 1) * 2048].copy_(_block((2048, TP_H), 40000 + b, 1.0))
    wg = torch.empty(fr, TP_H, dtype=torch.float16, device=dev)
    wu = torch.empty(fr, TP_H, dtype=torch.float16, device=dev)
    for j in range(nb):
        wg[j * TP_BLOCK:(j + 1) * TP_BLOCK].copy_(_block((TP_BLOCK, TP_H), 10000 + b0 + j, 0.02))
        wu[j * TP_BLOCK:(j + 1) * TP_BLOCK].copy_(_block((TP_BLOCK, TP_H), 20000 + b0 + j, 0.02))
    wd_cols = torch.cat([_block((TP_H, TP_BLOCK), 30000 + b0 + j, 0.02) for j in range(nb)], dim=1)
    wd = torch.empty(TP_H, fr, dtype=torch.float16, device=dev)
    wd.copy_(wd_cols.contiguous())
    del wd_cols
    torch.cuda.synchronize()
    return x, wg, wu, wd


def rows_owned(mode, rank, world):
    """Rows of the full output that a rank's result holds: all of them for the
    all-reduce, its own block [r T/N, (r+1) T/N) otherwise."""
    if mode == "allreduce" or world == 1:
        return 0, TP_T
    return rank * TP_T // world, (rank + 1) * TP_T // world


# ---- tensor-parallel MLP: parity --------------------------------------------------

def f16_ulp(a):
    """Spacing of binary16 at |a| (2^-24 below the normal range)."""
    import numpy as np
    a = np.abs(np.asarray(a, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def tp_parity(rank, world, x, wg, wu, wd, outs, dist):
    """Checks of this rank's results against the oracle (see module doc).
    outs: {mode: the result tensor that mode returned}."""
    import numpy as np
    import torch
    from oracle import oracle as O
    from torch_kunlun_b200 import ops
    S = 32
    r0 = rank * TP_T // world
    ax = ops.amax(x)
    gate = ops.linear_scaled(x, wg, amax_x=ax)
    up = ops.linear_scaled(x, wu, amax_x=ax)
    h = ops.silu_mul(gate, up)
    ah, awd = ops.amax(h), ops.amax(wd)
    res = {"rank": rank}
    # (1) the column-parallel GEMMs on sampled rows: bit-exact
    axv = np.float32(ax.cpu().item())
    xs = x[r0:r0 + S].cpu().numpy()
    ok = True
    for name, w, got in (("gate", wg, gate), ("up", wu, up)):
        wn = w.cpu().numpy()
        awn = O.amax(wn)
        want = O.epilogue(O.gemm_i16_strided(O.quant(xs, axv), O.quant(wn, awn).T), axv, awn, np.float16)
        g = got[r0:r0 + S].cpu().numpy()
        same = bool(np.array_equal(g.view(np.uint16), want.view(np.uint16)))
        res[f"{name}_bitexact"] = same
        ok = ok and same
    # (2) the SiLU gate: T(T(silu(gate)) * up) against float64 silu, <= 2 ulp16
    gs, us = gate[r0:r0 + S].cpu().numpy(), up[r0:r0 + S].cpu().numpy()
    want_h = O.silu_mul(gs, us)
    hs = h[r0:r0 + S].cpu().numpy()
    err = np.abs(hs.astype(np.float64) - want_h.astype(np.float64))
    h_ok = bool(np.all(err <= 2 * f16_ulp(want_h)))
    res["silu_gate_within_2ulp"] = h_ok
    res["silu_gate_differing_fraction"] = float(np.mean(hs.view(np.uint16) != want_h.view(np.uint16)))
    ok = ok and h_ok
    # (3) this rank's partial of the down projection on sampled rows: bit-exact
    ahv, awdv = np.float32(ah.cpu().item()), np.float32(awd.cpu().item())
    partial_s = ops.linear_scaled(h[r0:r0 + S], wd, amax_x=ah, amax_w=awd).cpu().numpy()
    want_p = O.epilogue(O.gemm_i16_strided(O.quant(hs, ahv), O.quant(wd.cpu().numpy(), awdv).T),
                        ahv, awdv, np.float16)
    same = bool(np.array_equal(partial_s.view(np.uint16), want_p.view(np.uint16)))
    res["down_partial_bitexact"] = same
    ok = ok and same
    # (4) the reduced rows against the rank-ordered fp32 sum of every rank's partial
    S2 = 64
    if world == 1:
        for mode, out in outs.items():
            got = out[:S].cpu().numpy()
            res[f"reduced_{mode}"] = "bitexact" if np.array_equal(got.view(np.uint16), want_p.view(np.uint16)) \
                else "FAIL"
            ok = ok and res[f"reduced_{mode}"] == "bitexact"
    else:
        partial = ops.linear_scaled(h, wd, amax_x=ah, amax_w=awd)
        tp_rows = TP_T // world
        sample = torch.cat([partial[q * tp_rows:q * tp_rows + S2] for q in range(world)]).contiguous()
        gathered = torch.empty(world * world * S2, TP_H, dtype=torch.float16, device=x.device)
        dist.all_gather_into_tensor(gathered, sample)
        parts = gathered.cpu().numpy().astype(np.float32).reshape(world, world, S2, TP_H)[:, rank]
        acc = np.zeros((S2, TP_H), dtype=np.float32)
        for r in range(world):
            acc = acc + parts[r]
        want = acc.astype(np.float16)
        bound = world * 2.0 ** -11 * np.abs(parts.astype(np.float64)).sum(0) + 2.0 ** -24
        for mode, out in outs.items():
            o0, _ = rows_owned(mode, rank, world)
            got = out[r0 - o0:r0 - o0 + S2].cpu().numpy()
            if np.array_equal(got.view(np.uint16), want.view(np.uint16)):
                v = "bitexact"
            elif np.all(np.abs(got.astype(np.float64) - want.astype(np.float64)) <= bound):
                v = "within_fp16_sum_bound"
            else:
                v = "FAIL"
            res[f"reduced_{mode}"] = v
            ok = ok and v != "FAIL"
            if mode.startswith("peer"):  # rank-ordered fp32 sum, one rounding: must be exact
                ok = ok and v == "bitexact"
        del partial, sample, gathered
    res["ok"] = bool(ok)
    del gate, up, h
    return res


# ---- tensor-parallel MLP: end to end ----------------------------------------------

def tp_e2e(x_host_rows, wg, wu, wd, dev, kunlun, dist, world, mode, steps, warmup, comm):
    """Steps through the public API with host buffers, pipelined as a serving
    loop runs them: each rank copies its row block of x from pinned host
    memory (a copy stream, two buffer sets), the ranks all-gather x over
    NVLink, run the MLP, and each copies its result rows back to pinned host
    memory (a third stream).  Device time of the whole loop / steps."""
    import torch
    from torch_kunlun_b200 import tp
    comp = kunlun.current_stream(dev)
    h2d, d2h = kunlun.Stream(dev), kunlun.Stream(dev)
    rows = x_host_rows.shape[0]
    xs = [torch.empty(rows, TP_H, dtype=torch.float16, device=dev) for _ in range(2)]
    xf = [torch.empty(TP_T, TP_H, dtype=torch.float16, device=dev) for _ in range(2)] if world > 1 else xs
    o0, o1 = rows_owned(mode, 0, world)
    out_rows = o1 - o0
    yh = [torch.empty(out_rows, TP_H, dtype=torch.float16).pin_memory() for _ in range(2)]
    freed, fetched = [None, None], [None, None]

    def step(i):
        s = i % 2
        with kunlun.stream(h2d):
            if freed[s] is not None:
                h2d.wait_event(freed[s])
            xs[s].copy_(x_host_rows, non_blocking=True)
            arrived = kunlun.Event(device=dev)
            arrived.record(h2d)
        comp.wait_event(arrived)
        if world > 1:
            dist.all_gather_into_tensor(xf[s], xs[s])
        y = tp.tp_mlp_forward(xf[s], wg, wu, wd, reduce=mode, chunks=4, comm_stream=comm)
        done = kunlun.Event(device=dev)
        done.record(comp)
        freed[s] = done
        with kunlun.stream(d2h):
            d2h.wait_event(done)
            if fetched[s] is not None:
                d2h.wait_event(fetched[s])
            yh[s].copy_(y, non_blocking=True)
            y.record_stream(d2h)
            got = kunlun.Event(device=dev)
            got.record(d2h)
            fetched[s] = got

    for i in range(warmup):
        step(i)
    kunlun.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = kunlun.Event(enable_timing=True), kunlun.Event(enable_timing=True)
    e0.record(comp)
    h2d.wait_event(e0)
    d2h.wait_event(e0)
    for i in range(steps):
        step(i)
    comp.wait_stream(h2d)
    comp.wait_stream(d2h)
    e1.record(comp)
    kunlun.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return ms, int(x_host_rows.nbytes), int(yh[0].nbytes)


# Kernel launches of this library per MLP step (counted from the code path of
# tp.tp_mlp_forward): amax(x), quantise(x), amax and quantise of each of the
# gate / up weights, their two GEMMs, the SiLU gate (with its amax), amax of
# the down weight; then quantise(down weight) and, per row block of the down
# projection, quantise + GEMM (plus the slot sum of the peer exchanges).
def tp_launches(mode, world):
    base = 10
    if world == 1 or mode == "reduce_scatter":
        return base + 3
    if mode == "allreduce":
        return base + 1 + 4 * 2
    if mode == "peer":
        return base + 1 + world * 2 + 1
    if mode == "peer_fused":
        return base + 2 + 1
    return base + 3


# ---- reference / CPU baseline: the oracle on a token sample ------------------------

def oracle_tp_sample(x_rows, wg, wu, wd):
    """The oracle's CPU restatement of the MLP on a few tokens with the full
    (TP = 1) weights: per-tensor quantisation of every operand, exact integer
    GEMMs, the SiLU gate, the epilogues.  Returns (seconds, int16 ops)."""
    from oracle import oracle as O
    t0 = time.perf_counter()
    gate = O.linear(x_rows, wg)
    up = O.linear(x_rows, wu)
    h = O.silu_mul(gate, up)
    O.linear(h, wd)
    dt = time.perf_counter() - t0
    return dt, 3 * 2 * x_rows.shape[0] * TP_H * TP_F


def oracle_tp_data(rows=REF_ROWS):
    """The full (TP = 1) weights and `rows` tokens of x drawn on the host:
    the same shapes, distributions and 512-row blocks as tp_inputs (the
    host generator's stream differs from the device's)."""
    import numpy as np
    import torch

    def blk(shape, seed, scale):
        g = torch.Generator().manual_seed(seed)
        return (torch.randn(shape, generator=g) * scale).half().numpy()
    nb = TP_F // TP_BLOCK
    wg = np.concatenate([blk((TP_BLOCK, TP_H), 10000 + j, 0.02) for j in range(nb)])
    wu = np.concatenate([blk((TP_BLOCK, TP_H), 20000 + j, 0.02) for j in range(nb)])
    wd = np.ascontiguousarray(np.concatenate([blk((TP_H, TP_BLOCK), 30000 + j, 0.02) for j in range(nb)], 1))
    x = blk((rows, TP_H), 40000, 1.0)
    return x, wg, wu, wd


def run_reference(args):
    """The reference path on the host cores: the oracle port of the MLP on
    16 tokens with all weights per step (rank 0 only; other ranks exit)."""
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    x, wg, wu, wd = oracle_tp_data(REF_ROWS)
    from oracle import oracle as O
    O.linear(x[:2, :64].copy(), wg[:8, :64].copy())  # build / warm the library
    for _ in range(max(1, args.warmup)):
        oracle_tp_sample(x, wg, wu, wd)
    times = []
    for _ in range(args.steps):
        dt, ops = oracle_tp_sample(x, wg, wu, wd)
        times.append(dt)
    ms = 1000 * statistics.mean(times)
    value = ops / (ms / 1000) / 1e12
    cores = threads_used()
    sample = (f"{REF_ROWS} of {TP_T} tokens through the whole MLP (TP = 1 weights: every weight amaxed and "
              "quantised per step) -- oracle: threaded C quantise, exact int64 GEMM, C epilogue")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, no dataset)",
        "config": {"workload": WORKLOAD, "sample": sample, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def threads_used():
    try:
        from oracle import oracle as O
        return int(O.lib().tko_num_threads())
    except Exception:
        return os.cpu_count() or 1


# ---- the single-GPU objects ----------------------------------------------------

def linear_object(dev, kunlun, flush, peaks, M, N, K, steps, warmup, with_e2e, cpu_sample):
    """One int16-quantised linear y = x W^T + b through torch.nn.functional.linear
    (step: amax + quantise + GEMM + epilogue), the GEMM kernel alone, and its
    roofline against the burst int16 peak."""
    import torch
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g).half()
    w = (torch.randn(N, K, generator=g) * 0.02).half()
    b = (torch.randn(N, generator=g) * 0.01).half()
    xd, wd, bd = x.to(dev), w.to(dev), b.to(dev)
    ops = 2 * M * N * K

    def step():
        torch.nn.functional.linear(xd, wd, bd)
    ts = timed_steps(step, steps, warmup, flush, kunlun)
    ms = sum(ts) / len(ts)
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    gemm = LimbGemm(xd, wd, out)
    gms = gemm.ms(kunlun, flush)
    traffic, tsrc = ncu_traffic(f"qgemm_linear_{M}x{N}x{K}.md")
    r = {"workload": f"int16-quantised linear x[{M},{K}] @ W[{N},{K}]^T + b, fp16",
         "ms_per_step": ms, "tops": ops / (ms / 1000) / 1e12, "gemm_kernel_ms": gms,
         "step_breakdown_ms": {"gemm": gms, "amax_quantise_and_launches": ms - gms},
         "roofline": roofline("tensor", ops / (gms / 1000) / 1e12, peaks["int16_burst"], "TOPS",
                              int16_peak_source(peaks, "burst"), traffic, tsrc,
                              kernel="qgemm_tc_kernel", ops_per_launch=ops, launch_ms=gms),
         "l2": L2_NOTE}
    if with_e2e:
        xh, wh, bh = x.pin_memory(), w.pin_memory(), b.pin_memory()
        yh = [torch.empty(M, N, dtype=torch.float16).pin_memory() for _ in range(2)]
        e2e_ms = linear_e2e(xh, wh, bh, yh, dev, kunlun, steps, warmup)
        r["e2e"] = {"value": ops / (e2e_ms / 1000) / 1e12, "unit": "TOPS", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(xh.nbytes + wh.nbytes + bh.nbytes),
                    "d2h_bytes_per_step": int(yh[0].nbytes),
                    "timing": "pipelined steps (H2D, op, D2H on three streams), device time / steps"}
    if cpu_sample:
        from oracle import oracle as O
        rows = 256
        xs, wn, bn = x[:rows].numpy(), w.numpy(), b.numpy()
        O.linear(xs[:8, :64].copy(), wn[:16, :64].copy(), None)
        reps = []
        for _ in range(3):
            t0 = time.perf_counter()
            O.linear(xs, wn, bn)
            reps.append(time.perf_counter() - t0)
        r["cpu_baseline"] = {"value": 2 * rows * N * K / statistics.mean(reps) / 1e12, "unit": "TOPS",
                             "cores": threads_used(), "kind": "port",
                             "sample": f"{rows} of {M} rows of x with all of W per call, 3 calls"}
    return r


def linear_e2e(xh, wh, bh, yh, dev, kunlun, steps, warmup):
    """Device time per step of pipelined end-to-end linear calls."""
    import torch
    comp = kunlun.current_stream(dev)
    h2d, d2h = kunlun.Stream(dev), kunlun.Stream(dev)
    xe = [torch.empty(xh.shape, dtype=xh.dtype, device=dev) for _ in range(2)]
    we = [torch.empty(wh.shape, dtype=wh.dtype, device=dev) for _ in range(2)]
    be = [torch.empty(bh.shape, dtype=bh.dtype, device=dev) for _ in range(2)]
    read, fetched = [None, None], [None, None]

    def step(i):
        s = i % 2
        with kunlun.stream(h2d):
            if read[s] is not None:
                h2d.wait_event(read[s])
            xe[s].copy_(xh, non_blocking=True)
            we[s].copy_(wh, non_blocking=True)
            be[s].copy_(bh, non_blocking=True)
            arrived = kunlun.Event(device=dev)
            arrived.record(h2d)
        comp.wait_event(arrived)
        y = torch.nn.functional.linear(xe[s], we[s], be[s])
        done = kunlun.Event(device=dev)
        done.record(comp)
        read[s] = done
        with kunlun.stream(d2h):
            d2h.wait_event(done)
            if fetched[s] is not None:
                d2h.wait_event(fetched[s])
            yh[s].copy_(y, non_blocking=True)
            y.record_stream(d2h)
            got = kunlun.Event(device=dev)
            got.record(d2h)
            fetched[s] = got

    for i in range(warmup):
        step(i)
    kunlun.synchronize()
    e0, e1 = kunlun.Event(enable_timing=True), kunlun.Event(enable_timing=True)
    e0.record(comp)
    h2d.wait_event(e0)
    d2h.wait_event(e0)
    for i in range(steps):
        step(i)
    comp.wait_stream(h2d)
    comp.wait_stream(d2h)
    e1.record(comp)
    kunlun.synchronize()
    return e0.elapsed_time(e1) / steps


def bert_inputs():
    import torch
    from torch_kunlun_b200 import encoder
    g = torch.Generator().manual_seed(0)
    x = torch.randn(BERT_B, BERT_L, BERT_H, generator=g).half()
    w = encoder.init_weights(BERT_H, BERT_F, generator=g)
    mask = encoder.padding_mask(BERT_B, BERT_L, BERT_TAIL)
    return x, w, mask


def bert_object(dev, kunlun, flush, peaks, steps, warmup, cpu):
    """Encoder block forward: tokens/s, and each op's device time and roofline
    from an instrumented pass (events between the ops of one block)."""
    import torch
    import torch.nn.functional as F
    from torch_kunlun_b200 import encoder, ops
    from torch_kunlun_b200.kunlun.attention import scaled_dot_product_attention
    x, w, mask = bert_inputs()
    xd, wd, md = x.to(dev), w.to(dev), mask.to(dev)

    def block():
        encoder.encoder_block(xd, wd, md, heads=BERT_HEADS, eps=1e-12)
    ts = timed_steps(block, steps, warmup, flush, kunlun)
    ms = sum(ts) / len(ts)
    macs = encoder.encoder_block_macs(BERT_B, BERT_L, BERT_H, BERT_F)
    T, H, E = BERT_B * BERT_L, BERT_H, BERT_H // BERT_HEADS

    def parts():
        ev = [kunlun.Event(enable_timing=True) for _ in range(8)]
        ev[0].record()
        x2 = xd.reshape(T, H)
        qkv = ops.linear(x2, wd.w_qkv, wd.b_qkv)
        ev[1].record()
        q5 = qkv.view(BERT_B, BERT_L, 3, BERT_HEADS, E).permute(2, 0, 3, 1, 4)
        ctx = scaled_dot_product_attention(q5[0], q5[1], q5[2], attn_mask=md)
        ev[2].record()
        ctx = ctx.transpose(1, 2).reshape(T, H)
        a = ops.linear(ctx, wd.w_o, wd.b_o, residual=x2)
        ev[3].record()
        h = F.layer_norm(a, (H,), wd.ln1_w, wd.ln1_b, 1e-12)
        ev[4].record()
        f1 = ops.linear(h, wd.w_1, wd.b_1, act="gelu")
        ev[5].record()
        f2 = ops.linear(f1, wd.w_2, wd.b_2, residual=h)
        ev[6].record()
        F.layer_norm(f2, (H,), wd.ln2_w, wd.ln2_b, 1e-12)
        ev[7].record()
        return ev
    names = ["qkv_linear", "attention", "out_linear_residual", "layer_norm1", "ffn1_linear_gelu",
             "ffn2_linear_residual", "layer_norm2"]
    acc = {n: 0.0 for n in names}
    reps = 5
    for i in range(reps + 2):
        flush()  # cold L2, and ~80 us of device work that puts the host ahead
        ev = parts()
        kunlun.synchronize()
        if i >= 2:
            for j, n in enumerate(names):
                acc[n] += ev[j].elapsed_time(ev[j + 1]) / reps
    total = sum(acc.values())
    lin_ops = {"qkv_linear": 2 * T * H * 3 * H, "out_linear_residual": 2 * T * H * H,
               "ffn1_linear_gelu": 2 * T * H * BERT_F, "ffn2_linear_residual": 2 * T * BERT_F * H}
    per_op = {}
    for n in names:
        t = acc[n]
        o = {"ms": t, "share": t / total}
        if n in lin_ops:
            o["roofline"] = roofline("tensor", lin_ops[n] / (t / 1000) / 1e12, peaks["int16_burst"], "TOPS",
                                     int16_peak_source(peaks, "burst"), ops_per_launch=lin_ops[n],
                                     note="whole op: amax + quantise + GEMM + fused epilogue")
        elif n == "attention":
            aops = 2 * 2 * BERT_B * BERT_HEADS * BERT_L * BERT_L * E
            o["roofline"] = roofline("tensor", aops / (t / 1000) / 1e12, peaks["int16_burst"], "TOPS",
                                     int16_peak_source(peaks, "burst"), ops_per_launch=aops,
                                     note="quantise + statistics + output kernels")
        else:
            nbytes = 2 * 2 * T * H + 2 * 2 * H
            o["roofline"] = roofline("hbm", nbytes / (t / 1000) / 1e9, peaks["hbm_gbs"], "GB/s",
                                     f"measured copy bandwidth, {peaks['source']}", algorithmic_bytes=nbytes)
        per_op[n] = o
    r = {"workload": BERT_WORKLOAD, "tokens_per_s": T / (ms / 1000), "ms_per_block": ms,
         "effective_tops": 2 * macs / (ms / 1000) / 1e12, "steps": steps, "warmup": warmup,
         "per_op": per_op, "per_op_source": "instrumented pass, events between the ops (5 blocks)"}
    if cpu:
        tps, threads = bert_cpu_baseline()
        r["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads,
                             "kind": "torch CPU aten fp32 eager",
                             "sample": "1 of 32 sequences (512 tokens), median of 3"}
    return r


def bert_cpu_baseline(batch=1, reps=3):
    """torch CPU aten fp32 eager encoder block on `batch` sequences (all host
    threads): tokens/s."""
    import torch
    import torch.nn.functional as F
    x, w, mask = bert_inputs()
    x, mask = x[:batch].float(), mask[:batch].float()
    f = {k: v.float() for k, v in vars(w).items()}
    torch.set_num_threads(os.cpu_count() or 1)
    B, L, H, E = batch, BERT_L, BERT_H, BERT_H // BERT_HEADS

    def block():
        x2 = x.reshape(B * L, H)
        qkv = F.linear(x2, f["w_qkv"], f["b_qkv"]).view(B, L, 3, BERT_HEADS, E).permute(2, 0, 3, 1, 4)
        ctx = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], attn_mask=mask)
        ctx = ctx.transpose(1, 2).reshape(B * L, H)
        h = F.layer_norm(x2 + F.linear(ctx, f["w_o"], f["b_o"]), (H,), f["ln1_w"], f["ln1_b"], 1e-12)
        g = F.gelu(F.linear(h, f["w_1"], f["b_1"]))
        return F.layer_norm(h + F.linear(g, f["w_2"], f["b_2"]), (H,), f["ln2_w"], f["ln2_b"], 1e-12)

    block()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        block()
        ts.append(time.perf_counter() - t0)
    return B * L / statistics.median(ts), torch.get_num_threads()


def bmm_object(dev, kunlun, flush, peaks, steps=20, warmup=3):
    """Attention-score chain S = A @ B, P = softmax(S), O = P @ V for A
    [64,512,128], B [64,128,512], V [64,512,128] ~N(0,1), fp16 and fp32:
    composed from the quantised bmm and softmax ops, and the same chain
    through the fused attention kernels (scale 1, no mask)."""
    import torch
    import torch_kunlun
    out = {"workload": "S = A[64,512,128] @ B[64,128,512], P = softmax(S), O = P @ V[64,512,128]",
           "ops_per_step": BMM_OPS}
    for dt, name in ((torch.float16, "fp16"), (torch.float32, "fp32")):
        g = torch.Generator().manual_seed(0)
        a = torch.randn(BMM_B, BMM_M, BMM_E, generator=g).to(dt).to(dev)
        b = torch.randn(BMM_B, BMM_E, BMM_M, generator=g).to(dt).to(dev)
        v = torch.randn(BMM_B, BMM_M, BMM_E, generator=g).to(dt).to(dev)
        kt = b.transpose(1, 2)

        def composed():
            torch.bmm(torch.softmax(torch.bmm(a, b), -1), v)

        def fused():
            torch_kunlun.scaled_dot_product_attention(a, kt, v, scale=1.0)

        for label, fn in (("composed", composed), ("fused", fused)):
            ts = timed_steps(fn, steps, warmup, flush, kunlun)
            ms = sum(ts) / len(ts)
            tops = BMM_OPS / (ms / 1000) / 1e12
            out[f"{name}_{label}"] = {
                "ms": ms, "tops": tops,
                "roofline": roofline("tensor", tops, peaks["int16_burst"], "TOPS", int16_peak_source(peaks, "burst"),
                                     ops_per_launch=BMM_OPS, note="whole chain, every launch")}
    return out


def conv_inputs(case, seed=0):
    import torch
    name, C, F, H, k, pad, groups, has_bias = case
    g = torch.Generator().manual_seed(seed)
    x = torch.relu(torch.randn(CONV_N, C, H, H, generator=g)).half()
    fan_in = (C // groups) * k * k
    w = (torch.randn(F, C // groups, k, k, generator=g) * (2.0 / fan_in) ** 0.5).half()
    bias = (torch.randn(F, generator=g) * 0.01).half() if has_bias else None
    return x, w, bias


def conv_ops(case):
    name, C, F, H, k, pad, groups, has_bias = case
    OH = H + 2 * pad - k + 1
    return 2 * CONV_N * OH * OH * F * (C // groups) * k * k


def conv_object(dev, kunlun, flush, peaks, cpu, steps=20, warmup=3):
    """ResNet-50-stage conv2d shapes at batch 64 (NCHW fp16, Kaiming-normal
    weights, ReLU(N(0,1)) inputs): device time per conv (amax, quantise and
    the convolution kernels), int16 TOPS, algorithmic HBM bytes, and the
    roofline of the bound that applies (tensor for the GEMM-shaped
    convolutions, HBM for the depthwise one)."""
    import torch.nn.functional as F
    res = {"workload": "conv2d NCHW fp16 batch 64, Kaiming-normal weights, ReLU(N(0,1)) inputs"}
    cb = conv_cpu_baseline() if cpu else {}
    for case in CONV_CASES:
        name, C, Fo, H, k, pad, groups, has_bias = case
        x, w, b = conv_inputs(case)
        xd, wd = x.to(dev), w.to(dev)
        bd = b.to(dev) if b is not None else None

        def fn():
            F.conv2d(xd, wd, bd, padding=pad, groups=groups)

        ts = timed_steps(fn, steps, warmup, flush, kunlun)
        ms = sum(ts) / len(ts)
        OH = H + 2 * pad - k + 1
        ops = conv_ops(case)
        nbytes = (x.numel() + CONV_N * Fo * OH * OH + w.numel()) * 2 + (Fo * 2 if has_bias else 0)
        r = {"ms": ms, "tops": ops / (ms / 1000) / 1e12, "ops": ops, "algorithmic_bytes": nbytes,
             "gbs": nbytes / (ms / 1000) / 1e9}
        if groups > 1:
            r["roofline"] = roofline("hbm", r["gbs"], peaks["hbm_gbs"], "GB/s",
                                     f"measured copy bandwidth, {peaks['source']}", algorithmic_bytes=nbytes)
        else:
            r["roofline"] = roofline("tensor", r["tops"], peaks["int16_burst"], "TOPS",
                                     int16_peak_source(peaks, "burst"), ops_per_launch=ops,
                                     hbm_frac=r["gbs"] / peaks["hbm_gbs"])
        if name in cb:
            r["cpu_baseline_tops"] = cb[name]
        res[name] = r
    if cpu:
        res["cpu_baseline"] = "torch CPU aten fp32 on 4 of 64 images, all host threads"
    return res


def conv_cpu_baseline():
    import torch
    import torch.nn.functional as F
    torch.set_num_threads(os.cpu_count() or 1)
    res = {}
    for case in CONV_CASES:
        name, C, Fo, H, k, pad, groups, has_bias = case
        x, w, b = conv_inputs(case)
        x4, wf = x[:4].float(), w.float()
        bf = b.float() if b is not None else None
        F.conv2d(x4, wf, bf, padding=pad, groups=groups)
        t0 = time.perf_counter()
        for _ in range(3):
            F.conv2d(x4, wf, bf, padding=pad, groups=groups)
        dt = (time.perf_counter() - t0) / 3
        res[name] = conv_ops(case) * 4 / CONV_N / dt / 1e12
    return res


def rowops_object(dev, kunlun, flush, peaks, steps=20, warmup=3):
    """The HBM-bound kernels on their benchmark shapes: softmax over
    [64, 512, 512] fp16 (the cfg2 scores) and [384, 512, 512] (BERT's),
    layer_norm over [16384, 768] fp16, and the cfg1 operands' amax + quantise
    through the C ABI.  Algorithmic bytes: 2 + 2 per element for softmax and
    layer_norm (plus gamma / beta), 2 read (amax) + 2 read + 2 written (two
    limbs) per element for the quantise."""
    import torch
    from torch_kunlun_b200 import _capi as C
    g = torch.Generator().manual_seed(0)
    s = torch.randn(64, 512, 512, generator=g).half().to(dev)
    s4 = torch.randn(384, 512, 512, generator=g).half().to(dev)
    h = torch.randn(16384, 768, generator=g).half().to(dev)
    gamma = (1 + 0.1 * torch.randn(768, generator=g)).half().to(dev)
    beta = (0.1 * torch.randn(768, generator=g)).half().to(dev)
    x = torch.randn(M1, K1, generator=g).half().to(dev)
    w = (torch.randn(N1, K1, generator=g) * 0.02).half().to(dev)
    L = C.lib()
    ld = (K1 + 15) // 16 * 16
    la = torch.empty(2 * M1 * ld, dtype=torch.int8, device=dev)
    lb = torch.empty(2 * N1 * ld, dtype=torch.int8, device=dev)
    amax = torch.empty(2, dtype=torch.float32, device=dev)

    def quantise():
        st = kunlun.current_stream().stream_id
        C.check(L.tk_amax(0, x.data_ptr(), 1, 0, M1 * K1, amax.data_ptr(), st), "amax")
        C.check(L.tk_amax(0, w.data_ptr(), 1, 0, N1 * K1, amax.data_ptr() + 4, st), "amax")
        C.check(L.tk_quantize_limbs(0, x.data_ptr(), 1, M1, K1, 0, K1, 1, amax.data_ptr(), 0,
                                    la.data_ptr(), st), "q")
        C.check(L.tk_quantize_limbs(0, w.data_ptr(), 1, N1, K1, 0, K1, 1, amax.data_ptr() + 4, 0,
                                    lb.data_ptr(), st), "q")
    out = {}
    for name, fn, nbytes in (
            ("softmax_64x512x512", lambda: torch.softmax(s, -1), 4 * s.numel()),
            ("softmax_384x512x512", lambda: torch.softmax(s4, -1), 4 * s4.numel()),
            ("layer_norm_16384x768", lambda: torch.nn.functional.layer_norm(h, (768,), gamma, beta, 1e-12),
             4 * h.numel() + 4 * 768),
            ("quantise_cfg1_operands", quantise, 6 * (M1 * K1 + N1 * K1))):
        ts = timed_steps(fn, steps, warmup, flush, kunlun)
        ms = sum(ts) / len(ts)
        gbs = nbytes / (ms / 1000) / 1e9
        out[name] = {"ms": ms, "gbs": gbs, "algorithmic_bytes": nbytes,
                     "roofline": roofline("hbm", gbs, peaks["hbm_gbs"], "GB/s",
                                          f"measured copy bandwidth, {peaks['source']}",
                                          algorithmic_bytes=nbytes, frac_of_8tbs=gbs / 8000.0)}
    return out


# ---- the headline run ---------------------------------------------------------------

def run_tp(args):
    import torch
    import torch.distributed as dist
    import torch_kunlun  # noqa: F401
    from torch_kunlun_b200 import tp
    kunlun = torch_kunlun.kunlun
    rank, local_rank, world = dist_env()
    kunlun.set_device(local_rank)
    torch.cuda.set_device(local_rank)
    dev = torch.device("kunlun", local_rank)
    if world > 1:
        # the communicator's init log (ranks, devices, channels) stays visible,
        # whatever level the environment preset
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        dist.init_process_group("bkcl", timeout=datetime.timedelta(seconds=180))
    peaks = load_peaks()
    mode = args.reduce if world > 1 else "none"
    x, wg, wu, wd = tp_inputs(rank, world, dev)
    comm = kunlun.Stream(dev)

    def step_fn(m):
        return lambda: tp.tp_mlp_forward(x, wg, wu, wd, reduce=m if world > 1 else "allreduce", chunks=4,
                                         comm_stream=comm)

    if world > 1:
        dist.barrier()
    kunlun.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        times = timed_steps(step_fn(mode), args.steps, args.warmup, lambda: None, kunlun)
    kunlun.synchronize()
    if world > 1:
        dist.barrier()
    my = step_stats(times)

    # the other reductions, as objects (fewer steps)
    mode_ms = {}
    extra_modes = [m for m in ("allreduce", "reduce_scatter", "peer", "peer_fused")
                   if world > 1 and m != mode and not args.no_extra_modes]
    for m in extra_modes:
        ts = timed_steps(step_fn(m), min(args.steps, 10), 2, lambda: None, kunlun)
        mode_ms[m] = sum(ts) / len(ts)

    # the three GEMM kernels alone, for the roofline
    gate_out = torch.empty(TP_T, TP_F // world, dtype=torch.float16, device=dev)
    up_out = torch.empty_like(gate_out)
    g_ms = LimbGemm(x, wg, gate_out).ms(kunlun, lambda: None, iters=3, warmup=1)
    u_ms = LimbGemm(x, wu, up_out).ms(kunlun, lambda: None, iters=3, warmup=1)
    from torch_kunlun_b200 import ops as kops
    hbuf = kops.silu_mul(gate_out, up_out)  # the step's activation (scales of its own)
    del gate_out, up_out
    y_out = torch.empty(TP_T, TP_H, dtype=torch.float16, device=dev)
    d_ms = LimbGemm(hbuf, wd, y_out).ms(kunlun, lambda: None, iters=3, warmup=1)
    del hbuf, y_out

    # parity of this rank's results (outside every timed region)
    outs = {mode: step_fn(mode)()}
    for m in extra_modes:
        outs[m] = step_fn(m)()
    kunlun.synchronize()
    par = tp_parity(rank, world, x, wg, wu, wd, outs, dist)
    del outs

    # end to end through the public API with host buffers
    r0, r1 = rank * TP_T // world, (rank + 1) * TP_T // world
    x_host = x[r0:r1].cpu().pin_memory()
    e2e_ms, h2d_b, d2h_b = tp_e2e(x_host, wg, wu, wd, dev, kunlun, dist, world,
                                  mode if world > 1 else "allreduce", args.steps, args.warmup, comm)

    # gather per-rank figures
    mine = [my["mean"], my["min"], my["median"], my["max"], e2e_ms, g_ms, u_ms, d_ms,
            1.0 if par["ok"] else 0.0] + [mode_ms.get(m, 0.0) for m in extra_modes]
    if world > 1:
        t = torch.tensor(mine, dtype=torch.float32).to(dev)
        allr = torch.empty(world * len(mine), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(allr, t)
        rows = allr.cpu().view(world, len(mine)).tolist()
    else:
        rows = [mine]
    # every rank's parity record travels through the store
    pars = [par]
    if world > 1:
        store = dist.distributed_c10d._get_default_store()
        store.set(f"bench_parity/{rank}", json.dumps(par))
        dist.barrier()
        pars = [json.loads(store.get(f"bench_parity/{r}").decode()) for r in range(world)]

    cpu_base = None
    extras = {}
    if rank == 0 and world == 1:
        kunlun.synchronize()
        del x
        if not args.no_cpu_baseline:
            xr, wgr, wur, wdr = oracle_tp_data(REF_ROWS)
            oracle_tp_sample(xr[:2], wgr, wur, wdr)  # warm
            reps = [oracle_tp_sample(xr, wgr, wur, wdr) for _ in range(2)]
            cpu_base = {"value": reps[0][1] / statistics.mean(r[0] for r in reps) / 1e12, "unit": "TOPS",
                        "cores": threads_used(), "kind": "port",
                        "sample": f"{REF_ROWS} of {TP_T} tokens through the whole MLP with all (TP = 1) "
                                  "weights, 2 calls (oracle: threaded C quantise, exact int64 GEMM, C epilogue)"}
            del xr, wgr, wur, wdr
        if not args.no_extra:
            del wg, wu, wd
            kunlun.empty_cache()
            extras = single_gpu_objects(dev, kunlun, peaks, args)

    if rank == 0:
        ms = max(r[0] for r in rows)
        e2e = max(r[4] for r in rows)
        gemm_ms = [max(r[5] for r in rows), max(r[6] for r in rows), max(r[7] for r in rows)]
        gemm_ops = 3 * 2 * TP_T * TP_H * (TP_F // world)
        achieved = gemm_ops / (sum(gemm_ms) / 1000) / 1e12
        peak = peaks["int16_burst"]  # the GEMM kernels are timed alone
        line = {
            "metric": METRIC, "value": TP_OPS / (ms / 1000) / 1e12, "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int16",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights in 512-row blocks, no dataset)",
            "config": {"workload": WORKLOAD, "T": TP_T, "H": TP_H, "F": TP_F, "parallelism": f"tp{world}",
                       "reduce": mode, "overlap": OVERLAP.get(mode, "none (one GPU)"),
                       "l2": "inputs (x 256 MiB, weights 1.4 GiB over the ranks) larger than L2"},
            "roofline": roofline("tensor", achieved, peak, "TOPS", int16_peak_source(peaks, "burst"),
                                 *(ncu_traffic(f"qgemm_tp_mlp_gate_{TP_T}x{TP_F}x{TP_H}.md") if world == 1
                                   else (None, None)),
                                 kernel="qgemm_tc_kernel (gate, up, down GEMMs of one rank)",
                                 ops_per_step=gemm_ops, gemm_ms=gemm_ms,
                                 frac_of_sustained=achieved / peaks["int16_sustained"],
                                 step_frac_of_sustained=(gemm_ops / (ms / 1000) / 1e12) / peaks["int16_sustained"],
                                 note="achieved = the rank's GEMM ops / the three GEMM kernels' event-timed "
                                      "durations (max over ranks); traffic: DRAM bytes of one gate GEMM launch "
                                      "(16384 x 28672 x 8192, one GPU) from the committed ncu summary, null for "
                                      "the smaller per-rank shards of N > 1"),
            "e2e": {"value": TP_OPS / (e2e / 1000) / 1e12, "unit": "TOPS", "ms_per_step": e2e,
                    "h2d_bytes_per_step": h2d_b * world, "d2h_bytes_per_step": d2h_b * world,
                    "per_rank_bytes": {"h2d": h2d_b, "d2h": d2h_b},
                    "timing": "pipelined steps: each rank's x row block H2D from pinned memory, all-gather "
                              "over NVLink, the MLP, its result rows D2H; device time of the loop / steps, "
                              "max over ranks"},
            "gpu_launches": tp_launches(mode, world) * args.steps,
            "clocks": clocks.summary(),
            "per_rank_ms": [{"rank": i, "mean": r[0], "min": r[1], "median": r[2], "max": r[3]}
                            for i, r in enumerate(rows)],
            "parity_ok": all(p["ok"] for p in pars),
            "parity": pars,
            "cpu_baseline": cpu_base,
        }
        if extra_modes:
            line["reduce_modes"] = {
                m: {"ms_per_step": max(r[9 + i] for r in rows),
                    "value": TP_OPS / (max(r[9 + i] for r in rows) / 1000) / 1e12, "overlap": OVERLAP[m]}
                for i, m in enumerate(extra_modes)}
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        tp.release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def single_gpu_objects(dev, kunlun, peaks, args):
    import torch
    flush = make_flush(dev, kunlun)
    cpu = not args.no_cpu_baseline
    out = {"objects_note": "single-GPU configs measured after the headline; L2 " + L2_NOTE +
                           "; each object carries the SM clocks sampled while it ran"}
    jobs = [
        ("linear_2048x4096x4096",
         lambda: linear_object(dev, kunlun, flush, peaks, M1, N1, K1, args.steps, args.warmup, True, cpu)),
        ("linear_4096x4096x4096",
         lambda: linear_object(dev, kunlun, flush, peaks, 4096, 4096, 4096, args.steps, args.warmup, False, False)),
        ("bert_block", lambda: bert_object(dev, kunlun, flush, peaks, max(5, args.steps // 4), args.warmup, cpu)),
        ("bmm_attention_scores", lambda: bmm_object(dev, kunlun, flush, peaks)),
        ("conv_resnet50", lambda: conv_object(dev, kunlun, flush, peaks, cpu)),
        ("rowops", lambda: rowops_object(dev, kunlun, flush, peaks)),
    ]
    for name, fn in jobs:
        with ClockSampler(torch.cuda.current_device()) as clocks:
            r = fn()
        r["clocks"] = clocks.summary()
        out[name] = r
    out["int8_live_tops"] = measured_int8_peak_tops()
    return out


def measured_int8_peak_tops():
    """cuBLASLt int8 GEMM (torch._int_mm) at 8192^3, best of 5 (burst) --
    printed beside the roofline denominators, not used as one."""
    import torch
    n = 8192
    a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    torch.cuda.empty_cache()
    return 2 * n ** 3 / best / 1e9


OVERLAP = {
    "allreduce": "down projection in 4 row blocks, each block's all-reduce on a second stream",
    "reduce_scatter": "none: one down GEMM, then the bkcl (NCCL) reduce-scatter",
    "peer": "down projection one owner's row block at a time; each finished block is copied by a copy "
            "engine into its owner's buffer (CUDA IPC, NVLink) while the next block computes; a "
            "one-element all-reduce as the barrier, then each rank sums its slots in rank order (fp32)",
    "peer_fused": "the down GEMM's epilogue stores each tile into the owning rank's buffer over NVLink "
                  "(CUDA IPC), a one-element all-reduce as the barrier, then each rank sums its slots",
}


# ---- the single-workload lines (profiling) -------------------------------------------

def run_single(args):
    """--workload linear | bert | rowops: one object as its own line (one GPU)."""
    import torch
    import torch_kunlun  # noqa: F401
    kunlun = torch_kunlun.kunlun
    dev = torch.device("kunlun", 0)
    peaks = load_peaks()
    flush = make_flush(dev, kunlun)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        if args.workload == "linear":
            r = linear_object(dev, kunlun, flush, peaks, M1, N1, K1, args.steps, args.warmup, False, False)
        elif args.workload == "linear4096":
            r = linear_object(dev, kunlun, flush, peaks, 4096, 4096, 4096, args.steps, args.warmup, False, False)
        elif args.workload == "bert":
            r = bert_object(dev, kunlun, flush, peaks, args.steps, args.warmup, False)
        elif args.workload == "conv":
            r = conv_object(dev, kunlun, flush, peaks, False, args.steps, args.warmup)
        elif args.workload == "bmm":
            r = bmm_object(dev, kunlun, flush, peaks, args.steps, args.warmup)
        else:
            r = rowops_object(dev, kunlun, flush, peaks, args.steps, args.warmup)
    print(json.dumps({"workload": args.workload, "steps": args.steps, "warmup": args.warmup,
                      "clocks": clocks.summary(), **r}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kunlun", choices=["kunlun", "reference"])
    ap.add_argument("--workload", default="tp_mlp",
                    choices=["tp_mlp", "linear", "linear4096", "bert", "conv", "bmm", "rowops"])
    ap.add_argument("--reduce", default="peer",
                    choices=["allreduce", "reduce_scatter", "peer", "peer_fused"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the single-GPU objects on the N=1 line")
    ap.add_argument("--no-extra-modes", action="store_true", help="time only the default reduction")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "tp_mlp":
        return run_tp(args)
    return run_single(args)


if __name__ == "__main__":
    sys.exit(main())
