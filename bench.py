#!/usr/bin/env python3
"""Benchmark of the b200q decode hot path (one JSON line on stdout, rank 0).

Workload (configs[1] of the benchmark configurations, the fused FFN block of a 4B-like layer): RMSNorm (eps 1e-6,
gain N(1, 0.1)) deferred into the Q8_0 quantizer, gate and up Q8_0 GEMVs [9216 x 2560] in one pass with the SwiGLU
epilogue, the down Q8_0 GEMV [2560 x 9216] with the residual ADD epilogue. The blocks are stacked as the layers of a model: L
blocks with distinct weights, each reading the residual stream the previous one wrote, form one command list of the
reference ISA (cut into lists of at most 128 commands between blocks), replayed as CUDA Graphs per step (one token
through the L-layer stack). L is chosen so that the
weights of one step exceed 3x the 126 MB L2, so every block reads weights that are not L2-resident. Synthetic seeded
weights with the config's distributions (no model files here).

metric: GEMV HBM GB/s = algorithmic bytes of the block (weights in their GGUF bits + x, gain, residual, y) per step
/ device time per step. N GPUs (torchrun): tensor parallel by default (each rank its F / N gate / up rows and down
columns, one ALLREDUCE of the block's output), or row-sharded with all-gathered outputs (--mp rows); the stack grows
with N so each GPU still reads > 3x its L2, and `value` = total algorithmic bytes / max-over-ranks time.

Beside the headline the line carries one object per other configuration, each measured on one GPU: `q4_0`
(configs[0], the standalone Q4_0 GEMV [9216 x 2560]), `kquant` (configs[2], Q5_K [9216 x 2560] and the Q6_K head),
`gdn_step` (configs[3], 128 sequential DeltaNet steps with conv1d, gates and the ssm_out Q4_0 GEMV) and `decode`
(configs[4], the 4B-like and 9B-like synthetic decoders, tokens/s).

--impl reference: the reference's own CPU arithmetic (fpga/src/gemvq_ref.h built from the reference sources into
oracle/_ref, OpenMP over row slices) on the same block and metric, on rank 0's host cores.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, F = 2560, 9216
EPS = 1e-6
XIN, GAIN, XN, FF, OUT = 0, H, 2 * H, 4 * H, 4 * H + F
PART = 5 * H + F  # tensor parallel: this rank's partial output of the down projection
RES = (XIN, OUT)  # the residual stream alternates between these two rows, layer by layer
ACT_FLOATS = 1 << 16
L2_BYTES = 126 << 20
DTYPE = "int8 x int8 -> int32, f32"  # exact integer block dots, FP32 terms and sums (the reference's arithmetic)
DATA = "synthetic (seeded GGUF Q8_0 weights of config 1)"


def load_package():
    name = "fpga_llama_gguf_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "fpga-llama-gguf_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def weight_bytes() -> int:
    return 2 * F * (H // 32) * 34 + H * (F // 32) * 34


def algorithmic_bytes() -> int:
    # weights in GGUF bits, x + gain read, residual read, y written
    return weight_bytes() + 4 * (H + H + H + H)


def gen_block(synth, seed: int):
    r = synth.rng(1, seed)
    return synth.q8_0(r, F, H), synth.q8_0(r, F, H), synth.q8_0(r, H, F)


def block_list(b2, hg, hu, hd, xin=XIN, out=OUT, world=1, rank=0):
    """One FFN block. Tensor parallel (world > 1): this rank's F / world rows of gate and up and the same columns of
    down give a partial output; rank 0 adds the residual, one ALLREDUCE sums the partials into `out`."""
    f = F // world
    head = [b2.rmsnorm(H, xin, GAIN, XN, EPS, flags=b2.NORM_DEFER),
            b2.gemv(b2.Q8_0, f, H, hg, XN, FF, b2.GEMV_SWIGLU), b2.gemv(b2.Q8_0, f, H, hu, XN, FF)]
    if world == 1:
        return b2.cmd_list(*head, b2.gemv(b2.Q8_0, H, F, hd, FF, out, b2.GEMV_ADD), b2.add(H, out, xin, out))
    down = ([b2.gemv(b2.Q8_0, H, f, hd, FF, PART, b2.GEMV_ADD), b2.add(H, PART, xin, PART)] if rank == 0
            else [b2.gemv(b2.Q8_0, H, f, hd, FF, PART)])
    return b2.cmd_list(*head, *down, b2.allreduce(H, PART, out))


def stack_list(b2, layers, upto=None, world=1, rank=0):
    """Command list of the layer stack (layer c: residual RES[c % 2] -> RES[(c + 1) % 2]); `upto` keeps only the
    first `upto` commands of each block (8 words each)."""
    return np.concatenate(stack_blocks(b2, layers, upto, world, rank))


def stack_blocks(b2, layers, upto=None, world=1, rank=0):
    parts = []
    for c, (hg, hu, hd) in enumerate(layers):
        cl = block_list(b2, hg, hu, hd, RES[c % 2], RES[(c + 1) % 2], world, rank)
        parts.append(cl[: upto * 8] if upto else cl)
    return parts


def stack_lists(b2, layers, upto=None, world=1, rank=0):
    """The stack as command lists of at most 128 commands (a list's limit), cut between blocks at the same blocks on
    every rank (as many blocks per list as rank 0's, the longest, fit): one step replays them in order, and the
    ranks' lists hold the same ALLREDUCEs (a collective's slot is its place in its list)."""
    blocks = stack_blocks(b2, layers, upto, world, rank)
    longest = max(c.size for c in stack_blocks(b2, layers[:1], upto, world, 0)) // 8
    per = max(1, b2.MAX_CMDS // longest)
    return [np.concatenate(blocks[i:i + per]) for i in range(0, len(blocks), per)]


def block_slices(mats, world: int, rank: int):
    """This rank's gate / up rows and down columns of the block's matrices (GGUF Q8_0 bytes)."""
    if world == 1:
        return [(mats[0], F, H), (mats[1], F, H), (mats[2], H, F)]
    f = F // world
    rows = slice(rank * f, (rank + 1) * f)
    down = np.ascontiguousarray(mats[2].reshape(H, F // 32, 34)[:, rank * f // 32:(rank + 1) * f // 32])
    return [(mats[0].reshape(F, -1)[rows], f, H), (mats[1].reshape(F, -1)[rows], f, H), (down.reshape(H, -1), H, f)]


class ClockSampler:
    """nvidia-smi samples (100 ms) over the whole GPU part of the run (the timed regions are short: a few ms for the
    stack), into a temporary file."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix="b200q_clocks_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()
        self.result = self._summary()
        try:
            os.unlink(self.path)
        except OSError:
            pass

    def summary(self):
        return getattr(self, "result", None) or self._summary()

    def _summary(self):
        try:
            rows = [ln.split(",") for ln in open(self.path).read().strip().splitlines() if ln.strip()]
        except Exception:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        pw = [float(r[3]) for r in rows if len(r) >= 9 and r[3].strip().replace(".", "").isdigit()]
        # under load: the samples whose power draw is in the upper half of the run's range (idle gaps between the
        # measurements, set-up and uploads excluded)
        busy = [c for c, p in zip(sm, pw) if pw and p >= (min(pw) + max(pw)) / 2] if len(pw) == len(sm) else sm
        return {"sm_mhz": statistics.median(busy or sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(busy),
                "power_w_max": max(pw) if pw else None,
                "window": "whole GPU part of the run, 100 ms samples"}


# the dominant kernel of the headline workload (the gate+up pass), as ncu names it in this build
TOP_KERNEL = "gemv_q8_kernel<8, 8, 2, 0>"


def profiled_traffic(kernel: str):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu summary of this build's kernels, or
    None when the summary has no capture of that kernel."""
    path = os.path.join(ROOT, "profiles", "gemv_q8_config1_full.txt")
    try:
        lines = open(path).read().splitlines()
    except OSError:
        return None
    for i, ln in enumerate(lines):
        if ln.startswith(f"--- {kernel}:"):
            for nxt in lines[i + 1:]:
                if nxt.startswith("---"):
                    break
                if nxt.strip().startswith("traffic_bytes_per_launch:"):
                    return int(nxt.split(":")[1].split()[0])
    return None


def measured_peak():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"], "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference(steps: int, warmup: int, budget_s: float, kind: str):
    """The reference CPU path on the host cores, on a bounded sample of the workload: the block's RMSNorm, three
    GEMVs, SwiGLU and residual add, each a vector call of the reference's own gemvq_ref.h compiled into oracle/_ref
    (the GEMVs parallel over row slices with OpenMP, all host threads), or of the restatement when that library is
    absent."""
    import ctypes
    import oracle
    sys.path.insert(0, ROOT)
    load_package()
    import fpga_llama_gguf_b200.synth as synth
    wg, wu, wd = gen_block(synth, 0)
    r = synth.rng(1, 99)
    x = synth.activation(r, H)
    gain = r.normal(1, 0.1, H).astype(np.float32)
    cores = os.cpu_count() or 1
    use_ref = kind == "reference" and oracle.ref_available()
    P = ctypes.c_void_p
    ptr = lambda a: a.ctypes.data_as(P)  # noqa: E731
    xn, g, u, h = (np.zeros(n, np.float32) for n in (H, F, F, F))
    d, y = np.zeros(H, np.float32), np.zeros(H, np.float32)

    def block():
        if use_ref:
            R = oracle.ref()
            R.ref_rmsnorm(ptr(x), ptr(gain), H, EPS, ptr(xn))
            R.ref_gemv_rows_omp(ptr(wg), ptr(xn), F, H, 8, ptr(g), cores)
            R.ref_gemv_rows_omp(ptr(wu), ptr(xn), F, H, 8, ptr(u), cores)
            R.ref_silu_mul(ptr(g), ptr(u), F, ptr(h))
            R.ref_gemv_rows_omp(ptr(wd), ptr(h), H, F, 8, ptr(d), cores)
            R.ref_add(ptr(d), ptr(x), H, ptr(y))
            return y
        xr = oracle.rownorm(x, gain, H, 1, EPS, 0)
        gg, _ = oracle.gemv(wg, xr, F, H, 8)
        uu, _ = oracle.gemv(wu, xr, F, H, 8)
        L = oracle.orc()
        hh = np.array([L.orc_silu_mul1(float(a), float(b), 0) for a, b in zip(gg, uu)], np.float32)
        return oracle.gemv(wd, hh, H, F, 8)[0] + x

    for _ in range(max(0, warmup)):
        block()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max(1, steps) and (time.perf_counter() < t_end or not times):
        t0 = time.perf_counter()
        block()
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    gbs = algorithmic_bytes() / per / 1e9
    what = ("gemvq_ref.h vector calls (rmsnorm, GEMV over OpenMP row slices, silu_mul, add)" if use_ref
            else "the oracle restatement")
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "cpu_model": cpu_model(),
            "kind": "reference" if use_ref else "port",
            "sample": f"{len(times)} FFN blocks (gate+up Q8_0 [9216x2560], down [2560x9216]) at {per * 1e3:.2f} ms "
                      f"each, {what}, {cores} threads"}


def timed_graph(ctx, torch, stream, cl, reps: int, warm: int = 5):
    """Device time (CUDA events on the library's stream) of one replay of list `cl` captured as a graph, in ms."""
    g = ctx.graph(cl)
    ctx.launch_many([g], warm)
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ctx.launch_many([g], reps)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    kernels = g.kernels
    g.close()
    return ms, kernels


def q4_0_bench(b2, torch, synth, dev: int, world: int) -> dict:
    """the standalone Q4_0 GEMV [9216 x 2560] against an fp32 N(0, 1) x quantized to Q8_0 inside the pass.
    One list holds 30 distinct copies of the matrix (398 MB, > 3x L2), consecutive GEMVs reading alternating x rows
    (so each is its own pass and quantizes its own x); GB/s of the GGUF weight bytes + x + y per GEMV."""
    if world > 1:
        return {"note": "measured on one GPU only"}
    peak, peak_kind = measured_peak()
    rows, cols, n = 9216, H, 30
    ctx = b2.Context(device=dev, weight_bytes=n * (b2.weight_device_bytes(rows, cols, b2.Q4_0) + (1 << 20)),
                     act_floats=1 << 20)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    r = synth.rng(0, 0)
    w = synth.q4_0(r, rows, cols)
    ctx.write(0, synth.activation(r, cols))
    ctx.write(cols, synth.activation(r, cols))
    cmds = []
    for i in range(n):
        hw = ctx.upload(w, rows, cols, b2.Q4_0)
        cmds.append(b2.gemv(b2.Q4_0, rows, cols, hw, (i % 2) * cols, 2 * cols + i * rows))
    ms, kernels = timed_graph(ctx, torch, stream, b2.cmd_list(*cmds), 50)
    ctx.close()
    per = w.nbytes + 4 * cols + 4 * rows
    us = ms * 1e3 / n
    gbs = per / (us * 1e-6) / 1e9
    return {"workload": "configs[0] Q4_0 GEMV [9216x2560], x quantized to Q8_0 in the pass", "us_per_gemv": round(us, 3),
            "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4), "peak_kind": peak_kind,
            "bytes_per_gemv": per, "copies": n, "kernels_per_gemv": kernels / n,
            "l2": f"{n} distinct copies ({n * w.nbytes >> 20} MiB) per list"}


def batch_bench(b2, torch, synth, dev: int, world: int) -> dict:
    """The GEMV_BATCH extension (the reference roadmap's batch path: one weight read for M activation rows) on the
    configs[0] matrix, Q4_0 [9216 x 2560]: one list of 30 distinct copies (> 3x L2), each a GEMV_BATCH of M rows;
    per M the time per command, the weight bytes per second and the activation rows per second (M / time)."""
    if world > 1:
        return {"note": "measured on one GPU only"}
    peak, peak_kind = measured_peak()
    rows, cols, n = 9216, H, 30
    ctx = b2.Context(device=dev, weight_bytes=n * (b2.weight_device_bytes(rows, cols, b2.Q4_0) + (1 << 20)),
                     act_floats=1 << 20)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    r = synth.rng(0, 1)
    w = synth.q4_0(r, rows, cols)
    xs = np.concatenate([synth.activation(r, cols) for _ in range(b2.BATCH_MAX)])
    ctx.write(0, xs)
    hs = [ctx.upload(w, rows, cols, b2.Q4_0) for _ in range(n)]
    out = {"workload": "GEMV_BATCH of Q4_0 [9216x2560] (configs[0] matrix), M activation rows per weight read",
           "copies": n, "peak_kind": peak_kind}
    y0 = b2.BATCH_MAX * cols
    for m in (1, 2, 4, 8):
        cl = b2.cmd_list(*[b2.gemv_batch(b2.Q4_0, rows, cols, h, 0, y0 + (i % 2) * m * rows, m) for i, h in enumerate(hs)])
        ms, kernels = timed_graph(ctx, torch, stream, cl, 30)
        us = ms * 1e3 / n
        gbs = w.nbytes / (us * 1e-6) / 1e9
        out[f"m{m}"] = {"us_per_command": round(us, 3), "weight_gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4),
                        "rows_per_s": round(m / (us * 1e-6), 1), "kernels_per_command": kernels / n}
    ctx.close()
    return out


def prefill_bench(b2, torch, synth, dev: int, world: int, batch8_rows_per_s: float | None) -> dict:
    """The prompt's matrix product on the tensor cores: a GEMV_BATCH command of T > 8 rows (tokens) runs as the token
    quantizer plus the tcgen05 GEMM (int8 MMA per 32-value block, FP32 block terms in block order, every output the
    GEMV's bits). Q4_0 [9216 x 2560] (the configs[0] matrix), 4 distinct copies per list, T = 128 and 512; per T the
    time per command, tokens per second (against the batch kernel's 8 rows per weight read) and the int8 MAC rate."""
    if world > 1:
        return {"note": "measured on one GPU only"}
    rows, cols, n = 9216, H, 4
    ctx = b2.Context(device=dev, weight_bytes=n * (b2.weight_device_bytes(rows, cols, b2.Q4_0) + (1 << 20)),
                     act_floats=1 << 24)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    r = synth.rng(0, 2)
    w = synth.q4_0(r, rows, cols)
    tmax = 512
    ctx.write(0, np.concatenate([synth.activation(r, cols) for _ in range(tmax)]))
    hs = [ctx.upload(w, rows, cols, b2.Q4_0) for _ in range(n)]
    out = {"workload": "GEMV_BATCH of T tokens x Q4_0 [9216x2560] (configs[0] matrix) on the tensor cores", "copies": n}
    y0 = tmax * cols
    for t in (128, tmax):
        cl = b2.cmd_list(*[b2.gemv_batch(b2.Q4_0, rows, cols, h, 0, y0 + (i % 2) * t * rows, t) for i, h in enumerate(hs)])
        ms, kernels = timed_graph(ctx, torch, stream, cl, 20)
        us = ms * 1e3 / n
        tok_s = t / (us * 1e-6)
        out[f"t{t}"] = {"us_per_command": round(us, 3), "tokens_per_s": round(tok_s, 1),
                        "int8_tops": round(2.0 * rows * cols * t / (us * 1e-6) / 1e12, 2),
                        "weight_gbs": round(w.nbytes / (us * 1e-6) / 1e9, 1), "kernels_per_command": kernels / n,
                        "vs_batch8": round(tok_s / batch8_rows_per_s, 2) if batch8_rows_per_s else None}
    ctx.close()
    return out


def gdn_bench(b2, torch, synth, dev: int, world: int, steps: int = 128) -> dict:
    """128 sequential Gated DeltaNet decode steps (hidden 2560, 16 heads, d_k = d_v = 128): the causal
    conv1d (k = 4) over the qkv projection with its 3-token state, the step with L2-normalized q / k, the gates from
    raw projections (beta = sigmoid, g = softplus(g + dt) * a), the gated RMSNorm * silu(z) output, and the ssm_out
    Q4_0 GEMV [2560 x 2048] with the residual add. 16 steps per list (one graph), replayed 8 times; the state
    [16, 128, 128] fp32 carries from step to step. Algorithmic bytes per step count the state read and written once,
    the ssm_out weights and the vectors; the 2 MiB state stays L2-resident across steps, so the latency per step is
    the number to read (GB/s beside it)."""
    if world > 1:
        return {"note": "measured on one GPU only"}
    peak, peak_kind = measured_peak()
    hv = hk = 16
    S = 128
    r = synth.rng(3, 0)
    ctx = b2.Context(device=dev, weight_bytes=64 << 20, act_floats=1 << 17, state_rows=hv * S)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    w_out = synth.q4_0(r, H, hv * S)
    h_out = ctx.upload(w_out, H, hv * S, b2.Q4_0, block_cols=256)
    QKV, CW, CS, QKVC = 0, 6144, 30720, 49152
    G, B, DT, A, Z, WN, Y, RES = 55296, 55312, 55328, 55344, 55360, 57408, 57536, 59584
    act = np.zeros(1 << 17, np.float32)
    act[QKV:QKV + 6144] = r.normal(0, 1, 6144)
    act[CW:CW + 4 * 6144] = r.normal(0, 0.5, 4 * 6144)
    act[CS:CS + 3 * 6144] = r.normal(0, 1, 3 * 6144)
    act[G:G + 32] = r.normal(0, 1, 32)
    act[DT:DT + 16] = r.normal(0, 1, 16)
    act[A:A + 16] = -np.exp(r.normal(0, 0.5, 16))
    act[Z:Z + 2048] = r.normal(0, 1, 2048)
    act[WN:WN + 128] = r.normal(1, 0.1, 128)
    act[RES:RES + H] = r.normal(0, 1, H)
    ctx.write(0, act)
    ctx.write_state(0, r.normal(0, 0.1, hv * S * S).astype(np.float32))
    per_list = 16
    cmds = []
    for t in range(per_list):
        # the residual stream alternates between two rows, step by step
        res_in, res_out = (RES, RES + H) if t % 2 == 0 else (RES + H, RES)
        cmds += [b2.conv(6144, QKV, CW, QKVC, CS, CS, True),
                 b2.gdn(hv, hk, QKVC, QKVC + 2048, QKVC + 4096, G, B, Y, 0, 0, S ** -0.5,
                        flags=b2.GDN_L2_QK | b2.GDN_GATED | b2.GDN_GATES | b2.GDN_WITH_OUT,
                        w_off=WN, z_off=Z, dt_off=DT, a_off=A),
                 b2.gemv(b2.Q4_0, H, hv * S, h_out, Y, res_out, b2.GEMV_ADD), b2.add(H, res_out, res_in, res_out)]
    cl = b2.cmd_list(*cmds)
    reps = steps // per_list
    ms, kernels = timed_graph(ctx, torch, stream, cl, reps * 4)
    ctx.close()
    us = ms * 1e3 / per_list
    # algorithmic bytes per step as the configuration's scope counts them: the state read and written once
    # (2 x 1 MiB), the ssm_out weights in their GGUF bits (2,949,120) and the step's vectors (200,832)
    per = 2 * hv * S * S * 4 + w_out.nbytes + 200_832
    gbs = per / (us * 1e-6) / 1e9
    return {"workload": "configs[3] GDN step + conv1d + gates + gated norm + ssm_out Q4_0 [2560x2048] + residual",
            "steps": reps * 4 * per_list, "us_per_step": round(us, 3), "bytes_per_step": per, "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "peak_kind": peak_kind, "kernels_per_step": kernels / per_list,
            "note": "the 2 MiB state is L2-resident across steps: latency per step is the figure of merit"}


def kquant_bench(b2, torch, synth, dev: int, world: int, max_over_ranks, barrier) -> dict:
    """the Q5_K GEMV [9216 x 2560] and the Q6_K output head [151936 x 2560] (three GEMV pieces on one x),
    against a Q8_K-quantized N(0, 1) x. The Q5_K matrix fits in L2, so a list holds 24 distinct copies whose
    consecutive GEMVs read alternating x rows (one pass each); the head reads 320 MB per pass. CUDA events on the
    library's stream; GB/s of the weights in their GGUF bits + x + y."""
    peak, _ = measured_peak()
    out = {}
    ctx = b2.Context(device=dev, weight_bytes=1200 << 20, act_floats=1 << 20)
    if world > 1:
        ctx.close()
        return {"note": "measured on one GPU only"}
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    r = synth.rng(2, 0)
    H = 2560
    ctx.write(0, synth.activation(r, H))
    ctx.write(H, synth.activation(r, H))

    def timed(cl, bytes_per_rep, passes):
        g = ctx.graph(cl)
        ctx.launch_many([g], 5)
        ctx.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.launch_many([g], 50)
        e1.record(stream)
        e1.synchronize()
        us = max_over_ranks(e0.elapsed_time(e1) / 50 * 1e3) / passes
        g.close()
        gbs = bytes_per_rep / passes / (us * 1e-6) / 1e9
        return {"us_per_pass": round(us, 2), "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}

    w5 = synth.q5_k(r, 9216, H)
    n5 = 24
    cmds = []
    for i in range(n5):
        h = ctx.upload(w5, 9216, H, 13)
        cmds.append(b2.gemv(13, 9216, H, h, (i % 2) * H, 4 * H + (i % 2) * 9216))
    q5 = timed(b2.cmd_list(*cmds), n5 * (w5.nbytes + 4 * H + 4 * 9216), n5)
    out["q5k_9216x2560"] = dict(q5, bytes_per_pass=w5.nbytes + 4 * H + 4 * 9216, copies=n5)
    ctx.reset_weights()
    w6 = synth.q6_k(r, 151936, H)
    rb = b2.gguf_row_bytes(H, 14)
    cmds, r0 = [], 0
    while r0 < 151936:
        n = min(50688, 151936 - r0)
        h = ctx.upload(w6.reshape(-1)[r0 * rb:(r0 + n) * rb], n, H, 14)
        cmds.append(b2.gemv(14, n, H, h, 0, 4 * H + r0))
        r0 += n
    head_bytes = w6.nbytes + 4 * H + 4 * 151936
    out["q6k_head_151936x2560"] = dict(timed(b2.cmd_list(*cmds), head_bytes, 1), bytes_per_pass=head_bytes)
    ctx.close()
    return out


def decode_bench(b2, torch, dist, dev: int, world: int, rank: int, shape, label: str, tokens: int, warm: int,
                 max_over_ranks, barrier, mp: str = "tp"):
    """Batch-1 greedy decode of the synthetic hybrid model: `tokens` tokens at positions prefill ..
    prefill + tokens - 1, each one stream-ordered record write (position + RoPE row, page-locked), the replay of the
    token's lists (one CUDA Graph each) and a stream-ordered read of the argmax token; the device chains the tokens
    (ARGMAX -> next GET_ROW). Timed with CUDA events on the context stream (max over ranks); then the same loop with
    the host waiting for every token (a host-side sampler's pattern), wall clock."""
    import fpga_llama_gguf_b200.decode as D
    t_setup = time.perf_counter()
    tp = world > 1 and mp == "tp"
    m = D.HybridDecoder(shape, world=world, rank=rank) if tp else D.HybridDecoder(shape)
    ctx = b2.Context(device=dev, **m.context_config(world))
    if world > 1:
        obj = [b2.Context.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.comm_init(world, rank, obj[0], b2.COMM_EXPLICIT if tp else 0)
    m.load(ctx)
    graphs = [ctx.graph(cl) for cl in m.token_lists()]
    setup_s = time.perf_counter() - t_setup
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))
    n = max(tokens, warm)
    rec = torch.empty((n, D.RECORD), dtype=torch.float32).pin_memory()
    rec.copy_(torch.from_numpy(np.stack([m.record(shape.prefill + t) for t in range(n)])))
    out = torch.zeros((n, 2), dtype=torch.float32).pin_memory()
    row = D.RECORD * 4

    def run(k: int):
        for t in range(k):
            ctx.write_async(m.L.REC, rec.data_ptr() + t * row, D.RECORD)
            ctx.launch_many(graphs, len(graphs))
            ctx.read_async(m.L.TOK, out.data_ptr() + t * 8, 2)

    run(warm)
    ctx.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    run(tokens)
    end.record(stream)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / tokens)
    toks = [int(v) for v in out[:tokens, 0].numpy().view(np.uint32)]
    barrier()
    # host waits for each token before the next (synchronous write, replay, synchronous read)
    n_sync = min(tokens, 32)
    t0 = time.perf_counter()
    for t in range(n_sync):
        ctx.write(m.L.REC, rec[t].numpy())
        ctx.launch_many(graphs, len(graphs))
        ctx.read(m.L.TOK, 2)
    ms_sync = max_over_ranks((time.perf_counter() - t0) / n_sync * 1e3)
    kernels = sum(g.kernels for g in graphs)
    for g in graphs:
        g.close()
    ctx.close()
    bpt = shape.bytes_per_token()
    peak, peak_kind = measured_peak()
    return {"model": label, "tokens": tokens, "positions": f"{shape.prefill}..{shape.prefill + tokens - 1}",
            "tokens_per_s": round(1e3 / ms, 2), "ms_per_token": round(ms, 4),
            "tokens_per_s_host_synced": round(1e3 / ms_sync, 2), "bytes_per_token": bpt,
            "hbm_gbs": round(bpt / (ms * 1e-3) / 1e9, 1),
            "frac_of_peak": round(bpt / (ms * 1e-3) / 1e9 / (peak * world), 4), "peak_kind": peak_kind,
            "roofline_tokens_per_s": round(peak * world * 1e9 / bpt, 1), "lists_per_token": len(graphs),
            "kernels_per_token": kernels, "h2d_bytes_per_token": row, "d2h_bytes_per_token": 8,
            "first_tokens": toks[:8], "scaling": "strong", "setup_s": round(setup_s, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="b200q", choices=["b200q", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--decode", default="4b,9b", help="synthetic decode models to run after the GEMV stack "
                    "(comma list of 4b, 9b; empty for none)")
    ap.add_argument("--decode-tokens", type=int, default=128)
    ap.add_argument("--no-kquant", action="store_true", help="skip the configs[2] K-quant GEMV measurement")
    ap.add_argument("--no-extras", action="store_true", help="skip the configs[0] / configs[3] objects")
    ap.add_argument("--mp", default="tp", choices=["tp", "rows"],
                    help="multi-GPU split: tp = each rank its own heads / FFN rows / column slices with one ALLREDUCE "
                    "per projection (default); rows = every matrix row-sharded by the library, outputs all-gathered")
    ap.add_argument("--decode-only", action="store_true", help="run only the decode measurement (for profiling "
                    "runs); the line then carries the decode object and no GEMV metric")
    ap.add_argument("--prefill-only", action="store_true", help="run only the prefill GEMM measurement (for "
                    "profiling runs); the line then carries the prefill object and no GEMV metric")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    config = {"workload": "configs[1] fused FFN block: deferred RMSNorm -> Q8_0 gate+up (SwiGLU) -> Q8_0 down "
                          "(+residual), hidden 2560, FFN 9216, stacked as the layers of one decode step",
              "global_batch": 1, "seq_len": 1,
              "parallelism": ("1 GPU" if world == 1 else
                              f"tensor parallel x{world} (FFN rows / down columns, one ALLREDUCE per block)"
                              if args.mp == "tp" else f"row-sharded x{world} (outputs all-gathered)")}

    per_layer = weight_bytes() // world
    n_layers = min(40, max(2, int(np.ceil(3 * L2_BYTES / max(per_layer, 1)))))
    config["layers"] = n_layers
    config["l2"] = (f"{n_layers} layers with distinct weights per step ({n_layers * per_layer >> 20} MiB per GPU > "
                    f"3x L2)")

    if args.impl == "reference":
        if rank != 0:
            return 0
        cb = cpu_reference(args.steps, min(args.warmup, 1), args.cpu_budget, "reference")
        line = {"metric": "GEMV HBM GB/s", "value": cb["value"], "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(n_layers * algorithmic_bytes() / cb["value"] / 1e6, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "data": DATA,
                "config": config, "impl": "reference", "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    b2 = load_package()
    import fpga_llama_gguf_b200.synth as synth
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    import fpga_llama_gguf_b200.decode as D
    shapes = {"4b": (D.SHAPE_4B, "4B-like: 24 GDN + 8 gated GQA layers, hidden 2560, FFN 9216, vocab 151936, Q4_0 + "
                                 "Q6_K head, 512-token F16 KV"),
              "9b": (D.SHAPE_9B, "9B-like: as 4B-like with hidden 4096, FFN 12288")}

    def run_decodes():
        out = {}
        for key in [k for k in args.decode.split(",") if k]:
            shape, label = shapes[key]
            out[key] = decode_bench(b2, torch, dist, dev, world, rank, shape, label, args.decode_tokens,
                                    max(3, min(args.warmup, 16)), max_over_ranks, barrier, args.mp)
        return out

    if args.prefill_only:
        prefill = prefill_bench(b2, torch, synth, dev, world, None)
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": "prefill tokens/s", "n_gpus": world, "impl": "b200q", "mode": "prefill-only",
                              "data": "synthetic", "prefill": prefill}), flush=True)
        return 0

    if args.decode_only:
        decode = run_decodes()
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": "decode tokens/s", "n_gpus": world, "impl": "b200q", "mode": "decode-only",
                              "data": "synthetic", "decode": decode}), flush=True)
        return 0

    # n_layers: enough layers that one step reads more than 3x the L2
    ctx = b2.Context(device=dev, weight_bytes=n_layers * (per_layer + (8 << 20)) + (64 << 20), act_floats=ACT_FLOATS)
    tp = world > 1 and args.mp == "tp"
    tw, tr = (world, rank) if tp else (1, 0)  # the lists' tensor-parallel split (rows mode: one-rank lists)
    if world > 1:
        obj = [b2.Context.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.comm_init(world, rank, obj[0], b2.COMM_EXPLICIT if tp else 0)
    mats = gen_block(synth, 0)
    layers = [tuple(ctx.upload(m, rows, cols, b2.Q8_0) for m, rows, cols in block_slices(mats, tw, tr))
              for _ in range(n_layers)]
    stack = [ctx.graph(cl) for cl in stack_lists(b2, layers, world=tw, rank=tr)]
    r = synth.rng(1, 99)
    x = synth.activation(r, H)
    gain = r.normal(1, 0.1, H).astype(np.float32)
    ctx.write(XIN, x)
    ctx.write(GAIN, gain)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", dev))

    # clocks sampled from the warm-up to the end of the GPU measurements
    clk = ClockSampler(dev).__enter__()
    # warm-up
    ctx.launch_many(stack, args.warmup * len(stack))
    ctx.synchronize()
    barrier()
    # timed region: K steps (each a replay of the whole stack)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    ctx.launch_many(stack, args.steps * len(stack))
    end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms)
    barrier()
    step_bytes = n_layers * algorithmic_bytes()
    value = step_bytes / (ms * 1e-3) / 1e9
    launches = sum(g.kernels for g in stack) * args.steps

    # roofline of the dominant kernel (the gate+up pass): the stack's gate+up passes alone, one graph, CUDA events
    peak, peak_kind = measured_peak()
    # per layer: norm + gate/up = one GEMV kernel
    ru = [ctx.graph(cl) for cl in stack_lists(b2, layers, upto=3, world=tw, rank=tr)]
    ctx.launch_many(ru, 5 * len(ru))
    ctx.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_ru = max(20, args.steps // 4)
    s2.record(stream)
    ctx.launch_many(ru, n_ru * len(ru))
    e2.record(stream)
    e2.synchronize()
    ru_ms = max_over_ranks(s2.elapsed_time(e2) / (n_ru * n_layers))
    ru_bytes = 2 * F * (H // 32) * 34 // world + 4 * (H + H)  # one rank's launch: its share of the rows
    achieved = ru_bytes / (ru_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None,
                "kernel": "gemv_q8_kernel (deferred RMSNorm + Q8_0 gate/up pair + SwiGLU)",
                "algorithmic_bytes_per_launch": ru_bytes, "us_per_launch": round(ru_ms * 1e3, 3),
                "peak_kind": peak_kind}
    traffic = profiled_traffic(TOP_KERNEL)
    if traffic is not None and tw > 1:
        # the capture is of the one-GPU launch (all 9216 rows); a tensor-parallel rank's launch streams its share of
        # the rows, and the launch's traffic is its weight stream, so it scales with the rows
        full_bytes = 2 * F * (H // 32) * 34 + 4 * (H + H)
        traffic = int(round(traffic * ru_bytes / full_bytes))
        roofline["traffic_note"] = "one-GPU capture scaled by this rank's share of the rows"
    roofline["traffic"] = traffic

    # end to end through the public API with host buffers: every step copies its x in from page-locked host memory
    # (stream-ordered b200q_act_write_async), replays the stack and copies y out (b200q_act_read_async); the host
    # waits once at the end (wall clock, max over ranks). Then the same loop with the host waiting for every step's
    # y before the next x (synchronous write / read, the reference's own call pattern), reported beside it.
    y_row = RES[n_layers % 2]
    e2e_steps = min(args.steps, 200)
    xin = torch.from_numpy(np.tile(x, (e2e_steps, 1))).pin_memory()
    yout = torch.empty((e2e_steps, H), dtype=torch.float32).pin_memory()
    ctx.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.write_async(XIN, xin.data_ptr() + i * 4 * H, H)
        for g in stack:
            g.launch()
        ctx.read_async(y_row, yout.data_ptr() + i * 4 * H, H)
    ctx.synchronize()
    t_e2e = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
    barrier()
    xs = xin[0].numpy()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.write(XIN, xs)
        for g in stack:
            g.launch()
        yout[i].numpy()[:] = ctx.read(y_row, H)
    t_sync = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
    e2e = {"value": round(step_bytes / t_e2e / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * H,
           "d2h_bytes_per_step": 4 * H, "ms_per_step": round(t_e2e * 1e3, 4),
           "host_synced": {"value": round(step_bytes / t_sync / 1e9, 2), "ms_per_step": round(t_sync * 1e3, 4)}}

    for g in stack + ru:
        g.close()
    ctx.close()

    q40 = gdn = batch = prefill = {}
    if not args.no_extras:
        q40 = q4_0_bench(b2, torch, synth, dev, world)
        gdn = gdn_bench(b2, torch, synth, dev, world)
        batch = batch_bench(b2, torch, synth, dev, world)
        prefill = prefill_bench(b2, torch, synth, dev, world, batch.get("m8", {}).get("rows_per_s"))
    decode = run_decodes()
    kquant = kquant_bench(b2, torch, synth, dev, world, max_over_ranks, barrier) if not args.no_kquant else {}
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    if dist:
        dist.destroy_process_group()

    cpu = None
    if rank == 0 and world == 1:
        try:
            cpu = cpu_reference(3, 1, min(args.cpu_budget, 20.0), "reference")
        except Exception as e:  # the CPU baseline is a reported number only
            cpu = {"value": None, "error": str(e)}
    if rank == 0:
        line = {"metric": "GEMV HBM GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "data": DATA, "config": config,
                "frac_of_peak": round(value / (peak * world), 4), "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches, "clocks": clocks, "q4_0": q40, "kquant": kquant, "gdn_step": gdn, "gemv_batch": batch,
                "prefill": prefill, "decode": decode}
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
