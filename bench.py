"""Benchmark of the ternary GEMV hot path (one JSON line on rank 0).

Workload (benchmark configuration 1, per-layer shape set at batch 1): a step is
one pass over a 64-layer model's ternary matmuls at batch 1. Every layer holds
its own resident weights of the seven config-1 shapes (q 5120->6144, k/v
5120->1024, o 6144->5120, gate/up 5120->17408, down 17408->5120; 5.8 GB in
all, 46x the 126 MB L2, so every step streams its weights from HBM and no L2
flush is needed) and runs the reference decoder's matmul call sequence
(src/cuda/gpu_decoder.cu:411-416, :437-450): quantise -> gemv[q,k,v] ->
quantise -> gemv+add[o] -> quantise -> gemv swiglu[gate,up] -> quantise ->
gemv+add[down]. Weights, scales and activations are seeded synthetic data with
the configuration's distributions (no checkpoint exists here).

value  = algorithmic HBM bytes of all launches / device time (GB/s), inputs resident.
e2e    = same metric through the same C-ABI calls with the step's activation
         inputs copied from pinned host memory and its outputs copied back,
         inside the timed region.
With --gpus N > 1 (torchrun), every matrix is N-sharded by rows across the
ranks (whole 8-row groups, shard.shard_rows) and each GEMV's output is
all-gathered in its epilogue over NVLink (tagged 64-bit stores into every
rank's buffer, btf_gemv_gather; no NCCL in the step); the total work is fixed,
so scaling is "strong".

The line also carries benchmark configuration 2 (the tcgen05 prefill GEMM, one
GPU) and configuration 3 (the 64-layer decode step as one CUDA graph; tensor
parallel at N > 1). On one GPU, `cpu_baseline` times the reference's CPU GEMV
and `decode_config3.cpu_baseline` its CPU emulator's decode step, both built
from the reference's sources into oracle/_ref, on bounded samples.

--impl reference times the reference's own CPU GEMV (oracle/_ref, built from
the reference sources; its emulator loop on all host threads) on a bounded
sample of the same workload, and adds its CPU emulator's decode step on
configuration 3's geometry (`decode_config3`, a bounded sample).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "bonsai-ternary-fast_b200")
sys.path.insert(0, PKG)

import synth  # noqa: E402

N_LAYERS = 64
METRIC = "ternary GEMV HBM GB/s, batch 1 (config-1 layer shape set, 64-layer step)"
UNIT = "GB/s"


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls NVML for SM clock and throttle reasons while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported, not required
            self.nv, self.err = None, str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.001)

    def start(self):
        if self.nv:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()

    def stop(self):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def report(self):
        if not self.nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "")}
        busy = [s for s in self.samples]
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(busy)}


# ------------------------------------------------------------------ CPU reference arm
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


_CPU_LAYER = {}


def cpu_reference(threads: int, reps: int = 3):
    """Times the reference's CPU GEMV (emulator loop, src/emu_decoder.cpp:143-165, compiled
    from the reference sources into oracle/_ref) on ONE layer of the workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    kind = "reference" if oracle.Reference.available() else "port"
    R = oracle.Reference() if kind == "reference" else None
    O = oracle.Oracle()
    if kind not in _CPU_LAYER:  # the layer's T2 matrices and Q8 activations, built once
        mats = {}
        for name, K, N in synth.LAYER_SHAPES:
            src = synth.ternary_ptq(N, K, seed=0)
            mats[name] = (R.repack_rows(src, N, K) if R else O.repack_t2(src, N, K)) + (K, N)
        acts = {K: (R or O).q8_rows(synth.activations(1, K, seed=2)) for K in (5120, 6144, 17408)}
        _CPU_LAYER[kind] = (mats, acts)
    mats, acts = _CPU_LAYER[kind]

    def one_layer():
        for name, (codes, scales, K, N) in mats.items():
            q, d, s = acts[K]
            if R:
                R.gemv(codes, scales, K, q, d, s, threads=threads)
            else:
                O.gemv(codes, scales, K, q, d, s, threads=threads)

    one_layer()  # warm caches / thread pool
    t0 = time.perf_counter()
    for _ in range(reps):
        one_layer()
    dt = (time.perf_counter() - t0) / reps
    layer_bytes = sum(synth.gemv_bytes(N, K) for _, K, N in synth.LAYER_SHAPES)
    return {"value": layer_bytes / dt / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"one of {N_LAYERS} layers (7 config-1 GEMVs, M=1), {reps} timed passes, "
                      f"{dt * 1e3:.1f} ms per layer", "cpu_model": cpu_model()}


def cpu_baseline_line(threads: int) -> dict:
    """The reference CPU GEMV on all host threads, plus the same sample on one thread."""
    cb = cpu_reference(threads)
    if threads > 1:
        one = cpu_reference(1, reps=1)
        cb["single_thread"] = {"value": one["value"], "unit": one["unit"], "sample": one["sample"]}
    return cb


def cpu_decode_reference(threads: int, steps: int = 3, geometry: dict | None = None) -> dict:
    """The reference's CPU emulator of its CUDA decode step (btf::make_emu_decoder,
    src/emu_decoder.cpp, compiled from the reference sources into oracle/_ref) on
    benchmark configuration 3's geometry, as a bounded sample: models with config
    3's widths and 4 and 8 layers (one and two periods of 3 delta-net layers + 1
    attention layer, plus the embedding and the 248320-row lm_head) are written
    with seeded weights, and each is timed over `steps` greedy steps after one
    warm-up step. The per-token time is linear in the layer count, so the 64-layer
    time is t4 + (t8 - t4) * 15. The context holds at most 5 tokens (the GPU
    bench's attention reads about 40; attention is a negligible share on the CPU).
    `geometry` replaces config 3's widths (tests use a small model)."""
    import shutil

    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    kind = "reference" if oracle.Reference.available() else None
    if kind is None:
        return {"unavailable": "oracle/_ref/libbtf_ref.so is not built"}
    R = oracle.Reference()
    base = geometry or CONFIG3
    per_tok = {}
    for n_layer in (4, 8):
        dims = dict(base, n_layer=n_layer)
        tensors = synth.qwen35_tensors(dims)
        need = sum(ne[0] // 128 * 28 * ne[1] if t == 143 else 4 * int(np.prod(ne)) for _, ne, t in tensors)
        dirs = [d for d in (os.environ.get("TMPDIR"), "/dev/shm", "/tmp", ROOT) if d and os.path.isdir(d)]
        room = [d for d in dirs if shutil.disk_usage(d).free > need * 1.25]
        if not room:
            return {"unavailable": f"no directory with {need * 1.25 / 1e9:.1f} GB free for the sample model"}
        path = os.path.join(room[0], f"btf_cpu_decode_{os.getpid()}_{n_layer}.gguf")
        try:
            synth.write_qwen35_gguf(path, dims, seed=3)
            em = oracle.Emulator(R, path, n_ctx=16, threads=threads)
            try:
                nxt, _ = em.step(1)
                t0 = time.perf_counter()
                for _ in range(steps):
                    nxt, _ = em.step(int(nxt))
                per_tok[n_layer] = (time.perf_counter() - t0) / steps
            finally:
                em.close()
        finally:
            if os.path.exists(path):
                os.remove(path)
    t64 = per_tok[4] + (per_tok[8] - per_tok[4]) * (base["n_layer"] - 4) / 4
    return {"value": 1.0 / t64, "unit": "tok/s", "s_per_token": t64, "cores": threads, "kind": kind,
            "sample": f"reference CPU emulator decode step at config-3 widths with 4 and 8 layers, {steps} timed "
                      f"steps each ({per_tok[4]:.3f} and {per_tok[8]:.3f} s per token), extrapolated linearly "
                      f"to {base['n_layer']} layers",
            "cpu_model": cpu_model()}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_threads()
    cb = cpu_reference(threads, reps=max(1, min(args.steps, 5)))
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "int8 x ternary",
            "data": "synthetic", "config": {"workload": "config1 layer set, batch 1, CPU emulator GEMV"},
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}, "vs_baseline": None}
    try:  # benchmark configuration 3 on the reference's CPU emulator (bounded sample)
        line["decode_config3"] = cpu_decode_reference(threads)
    except Exception as ex:
        line["decode_config3"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
class Model:
    """64 layers of resident panel weights (this rank's row shard of each matrix)."""

    def __init__(self, btf, torch, dev, rank, world):
        import shard

        self.shapes = {name: (K, N) for name, K, N in synth.LAYER_SHAPES}
        self.rows = {name: shard.shard_rows(N, world, rank) for name, (K, N) in self.shapes.items()}
        self.layers = []
        src = {}
        for name, (K, N) in self.shapes.items():
            r = self.rows[name]
            full = synth.ternary_ptq(N, K, seed=0)
            src[name] = torch.from_numpy(np.ascontiguousarray(full[r.r0:r.r0 + r.n])).to(dev)
        for _ in range(N_LAYERS):
            layer = {}
            for name, (K, N) in self.shapes.items():
                layer[name] = btf.repack_panels(src[name], self.rows[name].n, K)
            self.layers.append(layer)
        torch.cuda.synchronize()
        del src


def gpu_arm(args):
    import torch
    import torch.distributed as dist

    import btf_b200 as btf
    import shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    btf.kernels_init(local)
    model = Model(btf, torch, dev, rank, world)
    sh = model.shapes

    # activations and outputs (full width on every rank; each rank writes its row slice)
    xs = {k: torch.from_numpy(synth.activations(1, k, seed=2 + i)).to(dev)
          for i, k in enumerate((5120, 6144, 17408))}
    x_in = {"attn": xs[5120], "o": xs[6144], "ffn": xs[5120].clone(), "down": xs[17408]}
    acts = {k: btf.Q8Act.empty(1, sh_k, dev) for k, sh_k in (("attn", 5120), ("o", 6144), ("ffn", 5120),
                                                              ("down", 17408))}
    # full-width outputs; with N > 1 they live in a GatherArena: each rank's GEMV
    # stores its rows into every rank's copy over NVLink (btf_gemv_gather)
    outs = [n for n in sh if n != "up"]
    arena = None
    if world > 1:
        # tagged (value, tag) outputs: no counters or waits in the GEMV; one bounded
        # tag check per layer (btf_gather_wait) over the layer's six outputs
        # Per-layer output buffers, each stored exactly once per step, so the tag
        # only has to name the step (epoch; site 0 for every launch). The buffers
        # are 8*N bytes, multiples of 256, hence contiguous: one bounded tag check
        # over the whole range at the end of the step proves that every rank's
        # rows of every output have arrived (the inputs of this workload do not
        # depend on earlier outputs, so no launch waits for them sooner), and one
        # cross-rank barrier per step keeps every rank from storing into the next
        # step's buffers before all have checked this step's.
        arena = shard.GatherArena(btf, N_LAYERS * sum(8 * sh[n][1] for n in outs), world, rank, dev)
        offs = [{} for _ in range(N_LAYERS)]
        lay_out = [{} for _ in range(N_LAYERS)]
        for li in range(N_LAYERS):
            for n in outs:
                offs[li][n], lay_out[li][n] = arena.buffer((1, sh[n][1]), tagged=True)
        full_out = lay_out[N_LAYERS - 1]
        kind_names = (("qkv", ("q", "k", "v")), ("o", ("o",)), ("gateup", ("gate",)), ("down", ("down",)))
        gdesc = [{kind: arena.gather_desc([offs[li][n] + 8 * model.rows[n].r0 for n in names], tagged=True, site=0)
                  for kind, names in kind_names} for li in range(N_LAYERS)]
        total_words = N_LAYERS * sum(sh[n][1] for n in outs)
        assert offs[N_LAYERS - 1]["down"] + 8 * sh["down"][1] == 8 * total_words, "output buffers not contiguous"
        gwait_all = [(arena.word_ptr(0), total_words, 0)]
        gbar = arena.gather_desc([])
    else:
        full_out = {n: torch.zeros((1, sh[n][1]), device=dev) for n in outs}

    stream = torch.cuda.Stream(device=dev)

    # kernel end stamps (btf_stamp_next) in the timed graph: slot 8 * layer + k for
    # k = quantiser / GEMV of q,k,v | o | gate,up | down; they cost no event nodes,
    # so the programmatic-dependent-launch chain stays intact
    kinds = ("qkv", "o", "gateup", "down")
    stamps = torch.zeros(N_LAYERS * 8, dtype=torch.int64, device=dev)
    fstamps = torch.zeros(N_LAYERS * 4, dtype=torch.int64, device=dev)  # the fused path: one launch per GEMV

    def layer(L, li, stamped=False, fused=True):
        # fused: quantisation inside each GEMV (btf_gemv_f32, 4 launches per layer);
        # otherwise the drop-in pair launch_prep -> launch_gemv (8 launches per layer)
        def st_(k):
            if stamped:
                btf.stamp_next(stamps.data_ptr() + 8 * (8 * li + k))

        def gemv(segs, K, xk, mode, kind):
            ki = kinds.index(kind)
            if world > 1:  # drop-in pair with the all-gather in the GEMV epilogue
                st_(2 * ki)
                btf.quant_q8(x_in[xk], acts[xk], stream=stream)
                st_(2 * ki + 1)
                btf.launch_gemv_gather(segs, K, 1, acts[xk], mode, gdesc[li][kind], stream)
            elif fused:
                if stamped:
                    btf.stamp_next(fstamps.data_ptr() + 8 * (4 * li + ki))
                btf.launch_gemv_f32(segs, K, 1, x_in[xk], mode, stream)
            else:
                st_(2 * ki)
                btf.quant_q8(x_in[xk], acts[xk], stream=stream)
                st_(2 * ki + 1)
                btf.launch_gemv(segs, K, 1, acts[xk], mode, stream)

        def seg(n):
            r = model.rows[n]
            return (L[n], (lay_out[li] if world > 1 else full_out)[n][:, r.r0:], sh[n][1])

        gemv([seg("q"), seg("k"), seg("v")], 5120, "attn", btf.STORE, "qkv")
        gemv([seg("o")], 6144, "o", btf.ADD, "o")
        gemv([seg("gate"), (L["up"], None, 0)], 5120, "ffn", btf.SWIGLU, "gateup")
        gemv([seg("down")], 17408, "down", btf.ADD, "down")

    def step(fused=False, stamped=False):
        if world > 1:
            btf.gather_epoch_advance(arena.epoch_ptr, stream)
        for i, L in enumerate(model.layers):
            layer(L, i, stamped=stamped, fused=fused)
        if world > 1:  # every rank's rows of every output of the step have arrived
            btf.gather_wait(gwait_all, arena.epoch_ptr, stream)
            btf.gather_barrier(gbar, stream)

    # e2e variant: inputs from pinned host memory in, outputs back, every step
    h_in = {k: v.cpu().pin_memory() for k, v in x_in.items()}
    h_out = {k: torch.empty(v.shape, dtype=v.dtype).pin_memory() for k, v in full_out.items()}

    def step_e2e():
        for k in x_in:
            x_in[k].copy_(h_in[k], non_blocking=True)
        step()
        for k in full_out:
            h_out[k].copy_(full_out[k], non_blocking=True)

    h2d = sum(v.numel() * 4 for v in h_in.values())
    d2h = sum(v.numel() * 4 for v in h_out.values())

    # capture both variants as CUDA graphs (the reference replays its decode step as one graph)
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
            step(fused=True)
            step_e2e()
    torch.cuda.synchronize()
    # g_dev (timed, the headline) carries no instrumentation; g_stm is the same
    # step with the kernel end stamps, replayed separately for the per-kernel times
    g_dev, g_stm = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    g_e2e, g_unf = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_dev, stream=stream):
        step()
    with torch.cuda.graph(g_stm, stream=stream):
        step(stamped=True)
    with torch.cuda.graph(g_e2e, stream=stream):
        step_e2e()
    if world == 1:  # with N > 1 the step always runs the gathering pairs
        with torch.cuda.graph(g_unf, stream=stream):
            step(fused=True, stamped=True)
    torch.cuda.synchronize()

    def timed(graph, K, W):
        for _ in range(W):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(K):
                graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        torch.cuda.synchronize()
        return ms

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v for v in vis.split(",") if v.strip()]
    nvml_index = int(ids[local]) if local < len(ids) and ids[local].strip().isdigit() else local
    clocks = ClockSampler(nvml_index)
    clocks.start()
    ms_dev = timed(g_dev, args.steps, args.warmup)
    clocks.stop()
    ms_stm = timed(g_stm, args.steps, args.warmup)
    # exclusive time of each launch in the last stamped replay: its end minus the end
    # of the launch before it (layers 1..63; layer 0's first launch follows the
    # previous replay); the eight per-layer means add up to the layer time
    ends = stamps.cpu().numpy().astype(np.float64).reshape(N_LAYERS, 8)
    excl = np.diff(ends.reshape(-1))[7:].reshape(N_LAYERS - 1, 8) / 1e3  # us
    excl_us = excl.mean(axis=0)
    kern_ms = {k: excl_us[2 * i + 1] / 1e3 for i, k in enumerate(kinds)}  # the GEMV launches alone
    quant_ms = {k: excl_us[2 * i] / 1e3 for i, k in enumerate(kinds)}
    ms_e2e = timed(g_e2e, args.steps, args.warmup)
    ms_unf = timed(g_unf, args.steps, args.warmup) if world == 1 else None
    dev_err = btf.device_error()

    # algorithmic bytes (whole job: every matrix counted once)
    per_layer = {
        "qkv": sum(synth.gemv_bytes(sh[n][1], sh[n][0]) for n in ("q", "k", "v")) - 2 * 5120 * 5 // 4,
        "o": synth.gemv_bytes(sh["o"][1], sh["o"][0], add=True),
        "gateup": 2 * synth.gemv_bytes(sh["gate"][1], 5120) - 5120 * 5 // 4 - sh["gate"][1] * 4,
        "down": synth.gemv_bytes(sh["down"][1], sh["down"][0], add=True),
    }
    # path-independent bytes: x is read as fp32 (4 B/element) instead of the
    # Q8 copy (1.25 B/element) the two-kernel path hands between its kernels
    per_layer["qkv"] += 5120 * 11 // 4
    per_layer["o"] += 6144 * 11 // 4
    per_layer["gateup"] += 5120 * 11 // 4
    per_layer["down"] += 17408 * 11 // 4
    layer_bytes = per_layer["qkv"] + per_layer["o"] + per_layer["gateup"] + per_layer["down"]
    step_bytes = layer_bytes * N_LAYERS
    value = step_bytes * args.steps / (ms_dev * 1e-3) / 1e9
    e2e = step_bytes * args.steps / (ms_e2e * 1e-3) / 1e9
    fused_v = step_bytes * args.steps / (ms_unf * 1e-3) / 1e9 if ms_unf else None

    # each GEMV launch's own algorithmic bytes (codes + fp16 scales + Q8 activation + fp32 y,
    # y read too in add mode), for the per-kernel rates and the roofline
    kernel_bytes = {
        "qkv": sum(synth.gemv_bytes(sh[n][1], sh[n][0]) for n in ("q", "k", "v")) - 2 * 5120 * 5 // 4,
        "o": synth.gemv_bytes(sh["o"][1], sh["o"][0], add=True),
        "gateup": 2 * synth.gemv_bytes(sh["gate"][1], 5120) - 5120 * 5 // 4 - sh["gate"][1] * 4,
        "down": synth.gemv_bytes(sh["down"][1], sh["down"][0], add=True),
    }
    fused_kernels = None
    if ms_unf:
        fe = fstamps.cpu().numpy().astype(np.float64).reshape(-1)
        fx = (np.diff(fe)[3:].reshape(N_LAYERS - 1, 4) / 1e3).mean(axis=0)
        fused_kernels = {k: {"us": float(fx[i]), "GB/s": kernel_bytes[k] / (fx[i] * 1e-6) / 1e9}
                         for i, k in enumerate(kinds)}
        fused_kernels["sum_us_per_layer"] = float(fx.sum())
    peak, peak_kind = measured_peaks()
    # dominant kernel: the gate/up swiglu GEMV (52 % of the step's bytes); on this rank's shard
    dom_bytes = kernel_bytes["gateup"] / world
    dom_ach = dom_bytes / (kern_ms["gateup"] * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic_gateup_swiglu.txt")
    if os.path.exists(tpath):
        for line in open(tpath):
            if line.startswith("dram_bytes_per_launch:"):
                traffic = int(line.split(":")[1].strip()) // world
    kernels = {k: {"us": kern_ms[k] * 1e3, "GB/s": (kernel_bytes[k] / world) / (kern_ms[k] * 1e-3) / 1e9,
                   "quantiser_us": quant_ms[k] * 1e3,
                   "pair_GB/s": (kernel_bytes[k] / world) / ((kern_ms[k] + quant_ms[k]) * 1e-3) / 1e9}
               for k in kinds}
    kernels["sum_us_per_layer"] = float(excl_us.sum())
    kernels["layer_us_from_ms_per_step"] = ms_stm / args.steps * 1e3 / N_LAYERS
    kernels["ms_per_step_stamped"] = ms_stm / args.steps
    kernels["timing"] = ("exclusive time per launch in the stamped copy of the step graph: its end stamp "
                         "(btf_stamp_next: the last CTA's global timer) minus the previous launch's, mean over "
                         "layers 1..63 of the last of steps replays; no events between launches. The headline "
                         "value times the same graph without stamps")

    dec3 = lmh = None
    if world > 1:  # collective: the tensor-parallel decode step and the sharded lm_head on every rank
        dec3 = decode_config3(btf, torch, dev, world=world, rank=rank)
        try:
            lmh = lm_head_sharded(btf, torch, dev, world, rank)
        except Exception as ex:
            lmh = {"unavailable": f"{type(ex).__name__}: {ex}"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_dev / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x ternary (dp4a), fp32 accumulate",
            "data": "synthetic (seeded ternary weights, fp16 block-128 scales, N(0,1) activations)",
            "config": {"workload": "config1 per-layer shape set, batch 1, x64 layers per step",
                       "shapes": [f"{n}:{K}->{N}" for n, K, N in synth.LAYER_SHAPES],
                       "layers": N_LAYERS, "bytes_per_step": step_bytes,
                       "l2": "inputs larger than L2: 5.8 GB of distinct resident weights per step",
                       "parallelism": f"N-shard x{world}" + (", all-gather fused into the GEMV epilogue (NVLink "
                                                             "64-bit (value, tag) stores; one tag check of all "
                                                             "outputs per step; no NCCL in the step)"
                                                             if world > 1 else ""),
                       "graph": "one CUDA graph per step, programmatic dependent launch between kernels",
                       "path": "drop-in pairs: btf_quant_q8 (launch_prep) + btf_gemv (launch_gemv), PDL-chained"},
            "roofline": {"bound": "hbm", "achieved": dom_ach, "peak": peak, "unit": "GB/s",
                         "frac": dom_ach / peak, "traffic": traffic, "kernel": "gemv_kernel<1,SWIGLU> gate+up",
                         "bytes_per_launch": dom_bytes, "launch_us": kern_ms["gateup"] * 1e3,
                         "timing": "exclusive time of the gate+up GEMV launch inside the stamped copy of the "
                                   "step graph (its end stamp minus its quantiser's end stamp), mean over 63 "
                                   "layers; the eight launches of a layer add up to the layer time",
                         "peak_source": peak_kind, "frac_of_spec_8000": dom_ach / 8000.0},
            "kernels": kernels,
            "fused_quantise_path": {"value": fused_v, "unit": UNIT, "kernels": fused_kernels,
                                    "note": "btf_gemv_f32: quantisation inside "
                                    "each GEMV (4-CTA clusters), 4 launches per layer (same bytes counted)"}
            if world == 1 else None,
            "device_error_word": dev_err,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            # per step: 4 x (quantiser + GEMV) per layer; with N > 1 also the epoch
            # advance, one tag check of the step's outputs and the cross-rank barrier
            "gpu_launches": args.steps * (N_LAYERS * 8 + (3 if world > 1 else 0)),
            "clocks": clocks.report(),
        }
        if world == 1:
            try:
                line["reference_gpu_baseline"] = reference_gpu_baseline(torch, dev, step_bytes, args.steps,
                                                                         args.warmup)
                line["reference_gpu_baseline"]["product_over_reference"] = (
                    value / line["reference_gpu_baseline"]["value"])
            except Exception as ex:  # a baseline leg must not cost the product line
                line["reference_gpu_baseline"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
            line["prefill_gemm_config2"] = prefill_gemm(btf, torch, dev)
            line["decode_config3"] = decode_config3(btf, torch, dev)
            try:  # last of the GPU legs, so that a failure here costs only this entry
                line["lm_head_config4"] = lm_head_config4(btf, torch, dev)
            except Exception as ex:
                line["lm_head_config4"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
        else:
            line["decode_config3"] = dec3
            line["lm_head_config4"] = lmh
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_line(host_threads())
            try:
                line["decode_config3"]["cpu_baseline"] = cpu_decode_reference(host_threads())
            except Exception as ex:  # the GPU line must still print
                line["decode_config3"]["cpu_baseline"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
        print(json.dumps(line), flush=True)
    if world > 1:
        del g_dev, g_stm, g_e2e, g_unf
        torch.cuda.synchronize()
        dist.barrier()  # no rank still stores into another's arena
        arena.close()
        dist.barrier()
        dist.destroy_process_group()


def reference_gpu_baseline(torch, dev, step_bytes, steps, warmup):
    """The reference's OWN GPU matmul path on the same workload, as the GPU number to
    beat: its launch_prep (Q8 only) + launch_gemv (src/cuda/kernels.cu, built
    unmodified for sm_100a into oracle/_ref/libbtf_ref_gpu.so) over the same 64
    layers of config-1 weights, repacked to its T2 layout by its own launch_repack,
    in the same call order and captured as one CUDA graph per step (as its decoder
    captures its step). Same algorithmic bytes per step as the product's line."""
    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    if not oracle.ReferenceGPU.available():
        return {"unavailable": "oracle/_ref/libbtf_ref_gpu.so is not built (reference tree absent at build time)"}
    R = oracle.ReferenceGPU()
    R.init(dev.index)
    st = torch.cuda.Stream(device=dev)
    sh = {name: (K, N) for name, K, N in synth.LAYER_SHAPES}
    layer0 = {}
    for name, (K, N) in sh.items():
        src = torch.from_numpy(synth.ternary_ptq(N, K, seed=0)).to(dev)
        codes = torch.empty(N * K // 4, dtype=torch.uint8, device=dev)
        scales = torch.empty(N * K // 128, dtype=torch.int16, device=dev)
        R.repack(src.data_ptr(), N * K // 128, codes.data_ptr(), scales.data_ptr(), st.cuda_stream)
        layer0[name] = (codes, scales)
    torch.cuda.synchronize()
    layers = [layer0] + [{n: (c.clone(), s.clone()) for n, (c, s) in layer0.items()} for _ in range(N_LAYERS - 1)]
    xs = {k: torch.from_numpy(synth.activations(1, k, seed=2 + i)).to(dev) for i, k in enumerate((5120, 6144, 17408))}
    x_in = {"attn": xs[5120], "o": xs[6144], "ffn": xs[5120].clone(), "down": xs[17408]}
    acts = {k: (torch.empty(v.shape[1], dtype=torch.int8, device=dev),
                torch.empty(v.shape[1] // 32, dtype=torch.float32, device=dev),
                torch.empty(v.shape[1] // 32, dtype=torch.int32, device=dev)) for k, v in x_in.items()}
    ys = {n: torch.zeros((1, sh[n][1]), device=dev) for n in sh if n != "up"}

    def gemv(names, xk, mode):
        K = sh[names[0]][0]
        x = x_in[xk]
        q, d, s = acts[xk]
        R.quant(x.data_ptr(), K, 1, K, q.data_ptr(), d.data_ptr(), s.data_ptr(), st.cuda_stream)
        segs = []
        for n in names:
            c, sc = L[n]
            y = ys.get(n)
            segs.append((c.data_ptr(), sc.data_ptr(), sh[n][1], y.data_ptr() if y is not None else 0,
                         sh[n][1] if y is not None else 0))
        R.gemv(segs, K, 1, q.data_ptr(), d.data_ptr(), s.data_ptr(), mode, st.cuda_stream)

    def step():
        nonlocal L
        for L in layers:
            gemv(("q", "k", "v"), "attn", 0)
            gemv(("o",), "o", 1)
            gemv(("gate", "up"), "ffn", 2)
            gemv(("down",), "down", 1)

    L = None
    with torch.cuda.stream(st):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        step()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    with torch.cuda.stream(st):
        for _ in range(steps):
            g.replay()
    b.record(st)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    out = {"value": step_bytes / (ms * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": ms, "steps": steps,
           "kind": "reference", "path": "reference launch_prep (Q8) + launch_gemv, src/cuda/kernels.cu built "
                                          "unmodified for sm_100a, T2 weights from its launch_repack, one CUDA graph "
                                          "per step, same call order and bytes as the product line",
           "gpu_launches": steps * N_LAYERS * 8}
    del g, layers, layer0
    torch.cuda.empty_cache()
    return out


def lm_head_sharded(btf, torch, dev, world, rank, reps=10, replays=3):
    """Benchmark configuration 4's lm_head N-sharded over `world` GPUs (collective):
    K=5120 -> N=248320, rank r holding its rows (shard.shard_rows, whole 8-row
    groups; 338/world MB of panels), at batch 1 and 16, with the all-gather fused
    into the GEMV epilogue (btf_gemv_gather, tagged 64-bit stores into every rank's
    full-width output over NVLink; batch 16 runs on the weight-major tcgen05 GEMM
    with the same stores). One run: epoch advance, `reps` launches (each
    into its own output buffer), one bounded tag check of all the run's outputs,
    one cross-rank barrier; captured as a CUDA graph, CUDA events, max over ranks.
    GB/s = algorithmic bytes of the whole lm_head per launch (weights once, the Q8
    activation, the fp32 output) / time per launch: the aggregate over the ranks.
    The weights are the same 16-fold seeded block as lm_head_config4."""
    import torch.distributed as dist

    import shard

    _, K, N = synth.LM_HEAD
    r = shard.shard_rows(N, world, rank)
    full = torch.from_numpy(synth.ternary_ptq(N // 16, K, seed=7)).to(dev).repeat(16, 1)
    src = full[r.r0:r.r0 + r.n].contiguous()
    del full
    pm = btf.repack_panels(src, r.n, K)
    torch.cuda.synchronize()
    del src
    peak, peak_src = measured_peaks()
    st = torch.cuda.Stream(device=dev)
    out = {"shape": f"K{K}_N{N}", "n_gpus": world, "rows_per_gpu": r.per,
           "panel_bytes_per_gpu": btf.panel_bytes(r.n, K), "peak_per_gpu": peak, "peak_source": peak_src,
           "launches_per_run": reps}
    for M in (1, 16):
        arena = shard.GatherArena(btf, reps * M * N * 8, world, rank, dev)
        bufs = [arena.buffer((M, N), tagged=True) for _ in range(reps)]
        descs = [arena.gather_desc([off + 8 * r.r0], tagged=True, site=0) for off, _ in bufs]
        gwait_all = [(arena.word_ptr(bufs[0][0]), reps * M * N, 0)]
        gbar = arena.gather_desc([])
        act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=8)).to(dev))
        torch.cuda.synchronize()

        def run():
            btf.gather_epoch_advance(arena.epoch_ptr, st)
            for k in range(reps):
                btf.launch_gemv_gather([(pm, bufs[k][1][:, r.r0:], N)], K, M, act, btf.STORE, descs[k], st)
            btf.gather_wait(gwait_all, arena.epoch_ptr, st)
            btf.gather_barrier(gbar, st)

        with torch.cuda.stream(st):
            run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            run()
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        with torch.cuda.stream(st):
            for _ in range(replays):
                g.replay()
        b.record(st)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item()) * 1e3 / (replays * reps)
        nbytes = btf.panel_bytes(N, K) + M * (K + K // 32 * 8) + M * N * 4
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        # the routing rules of btf_gemv_gather (mma_serves, wm_serves)
        units = -(-r.n // 32)
        mma = K <= btf.GEMV_MMA_MAX_K and ((9 <= M <= 16 and units >= sms) or (5 <= M <= 8 and units >= 2 * sms)
                                           or (3 <= M <= 4 and units >= 8 * sms))
        wm = not mma and M >= 9 and -(-r.n // 128) >= sms * 2 // 3
        err = btf.device_error()
        out[f"M{M}"] = {"us": us, "GB/s": nbytes / (us * 1e-6) / 1e9,
                        "GB/s_per_gpu": nbytes / world / (us * 1e-6) / 1e9,
                        "frac_of_hbm_per_gpu": nbytes / world / (us * 1e-6) / 1e9 / peak,
                        "bytes_per_launch": nbytes,
                        "weight_passes": 1 if mma or wm else -(-M // btf.gemv_max_nb(K)),
                        "path": "btf_gemv_gather -> " + ("gemv_mma_kernel (warp int8 MMA, tagged stores)" if mma
                                                         else "gemm_wm_kernel (weight-major tcgen05, tagged stores)"
                                                         if wm else "gemv_kernel (tagged stores)"),
                        "device_error_word": err}
        del g
        torch.cuda.synchronize()
        dist.barrier()  # no rank still stores into another's arena
        arena.close()
        dist.barrier()
    return out


PREFILL_SHAPES = ((64, 5120, 17408), (512, 5120, 17408), (64, 17408, 5120), (512, 17408, 5120))

# Benchmark configuration 3: the 64-layer hybrid decoder (hidden 5120, FFN 17408,
# vocab 248320; 3 of 4 layers gated delta net, every 4th full GQA attention over
# a 4096-token fp16 KV cache), with the real model's per-head geometry (24 q / 4
# kv heads of 256, RoPE on 64 dims; delta net 16 k-heads / 48 v-heads of 128,
# inner 6144, conv 4) and Hadamard block 1024. Seeded random weights.
CONFIG3 = dict(n_layer=64, n_embd=5120, n_ff=17408, n_vocab=248320, n_head=24, n_head_kv=4, head_dim=256, n_rot=64,
               d_state=128, n_group=16, dt_rank=48, d_inner=6144, conv_kernel=4, hadamard_block=1024,
               rope_base=1e7, rms_eps=1e-6)


def decode_config3(btf, torch, dev, steps=64, warmup=8, n_ctx=4096, world=1, rank=0):
    """Benchmark configuration 3: batch-1 decode steps of the synthetic 64-layer
    decoder as one CUDA graph per token (btf_decoder_*). `value`: tokens/s of a
    device-side greedy loop (each step feeds its argmax to the next), CUDA events
    on the decoder's stream; `e2e`: the synchronous step API (token from the host,
    next token back). Roofline: bytes one token reads (resident weights, one
    embedding row, recurrent state read + written, K/V of the cached tokens).
    With world > 1 (collective) every matmul is N-sharded over the ranks
    (btf_decoder_synthetic_tp) and times are the max over ranks; the roofline
    is per GPU (this rank's bytes)."""
    if world > 1:
        import torch.distributed as dist
    dec = btf.Decoder(dims=CONFIG3, seed=3, n_ctx=n_ctx, device=dev.index, world=world, rank=rank)
    if world > 1:
        dec.connect_tp()
    info = dec.info()
    st = torch.cuda.ExternalStream(info["stream"], device=dev)

    def timed(fn, n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    dec.step(1)  # captures the graph
    dec.run(warmup)
    torch.cuda.synchronize()
    p0 = dec.info()["pos"]
    ms = timed(lambda: dec.run(steps), steps)
    ne2e = 16

    def e2e_steps():
        nxt = 1
        for _ in range(ne2e):
            nxt, _ = dec.step(nxt)

    ms_e2e = timed(e2e_steps, ne2e)
    err = btf.device_error()
    ctx_mean = p0 + (steps + 1) / 2.0  # cached tokens the timed steps read on average
    per_tok = info["weight_bytes"] + info["state_bytes"] + info["kv_bytes_per_token"] * ctx_mean
    gbs = per_tok / (ms * 1e-3) / 1e9
    peak, peak_src = measured_peaks()
    n_gdn = sum(1 for il in range(CONFIG3["n_layer"]) if (il + 1) % 4)
    out = {"metric": "decode tokens/s, batch 1 (config 3)", "value": 1e3 / ms, "unit": "tok/s", "ms_per_token": ms,
           "n_gpus": world, "steps": steps, "warmup": warmup + 1, "context_start": p0, "n_ctx": n_ctx,
           "config": dict(CONFIG3), "data": "synthetic (seeded ternary panels, uniform vectors)",
           "parallelism": "one GPU" if world == 1 else
           f"tensor parallel x{world}: every matmul N-sharded, outputs all-gathered in the GEMV epilogue "
           "(NVLink stores, counted completion); the rest replicated",
           "bytes_per_token_per_gpu": per_tok, "weight_bytes_per_gpu": info["weight_bytes"],
           "state_bytes": info["state_bytes"], "kv_bytes_per_cached_token": info["kv_bytes_per_token"],
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                        "peak_source": peak_src, "per": "GPU"},
           "e2e": {"value": 1e3 / ms_e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
           # per token: 9 launches per layer (prep + GEMV x 4, the mixer or the one attention
           # kernel), embed, final prep, lm_head, 2 argmax stages
           "gpu_launches_per_token": 9 * CONFIG3["n_layer"] + 5, "n_gdn_layers": n_gdn,
           "device_error_word": err, "path": "btf_decoder_run: one graph replay per token"}
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # no rank still stores into another's arena
    dec.close()
    if world > 1:
        dist.barrier()
    return out


def prefill_gemm(btf, torch, dev, reps=10):
    """Benchmark configuration 2: the tcgen05 prefill GEMM (btf_gemm) at M = 64 and 512
    on both weight shapes, each launch over one of 4 rotating weight copies (> L2),
    timed with CUDA events around a CUDA graph of `reps` launches. btf_gemm runs
    M = 64 over the 136 tiles of 5120 -> 17408 on the weight-major kernel and the
    other cases on the 128-row GEMM (`kernel` names which)."""
    out = {}
    for M, K, N in PREFILL_SHAPES:
        src = torch.from_numpy(synth.ternary_ptq(N, K, seed=0)).to(dev)
        mats = [btf.repack_panels(src, N, K) for _ in range(4)]
        act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=2)).to(dev))
        y = torch.empty((M, N), device=dev)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for i in range(4):
                btf.launch_gemm([(mats[i % 4], y, N)], K, M, act, btf.STORE, st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(reps):
                btf.launch_gemm([(mats[i % 4], y, N)], K, M, act, btf.STORE, st)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        with torch.cuda.stream(st):
            g.replay()
        b.record(st)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / reps
        ops = 2.0 * M * N * K
        tiles = -(-N // 128)
        out[f"M{M}_K{K}_N{N}"] = {"us": us, "TOPS": ops / us / 1e6,
                                  "frac_of_int8_spec_4500": ops / us / 1e6 / 4500.0,
                                  "weight_GBps": btf.panel_bytes(N, K) / us / 1e3,
                                  "kernel": "gemm_wm_kernel" if M <= 64 and tiles >= 148 * 2 // 3 else "gemm_kernel"}
        del g, mats, src
    return out


def lm_head_config4(btf, torch, dev, reps=20):
    """Benchmark configuration 4's lm_head on one GPU: the ternary GEMV K=5120 ->
    N=248320 (338 MB of panels, 2.7x L2) at batches 1, 8 and 16 through btf_gemv
    (batches 8 and 16 run on the warp-MMA GEMM, one pass over the weights; the
    4-row GEMV passes it replaced and, at batch 16, the tcgen05 weight-major GEMM
    are timed beside it), each launch over one of 2 weight copies, timed with
    CUDA events around a CUDA graph of `reps` launches.
    GB/s counts the algorithmic bytes (weights once, the Q8 activation, the fp32
    output); `weight_passes` is how often a launch streams the weights. The
    weights are 16 copies of one seeded 15520-row PTQ1_0 block with config 0's
    distributions (the number of bytes, not their values, sets the time)."""
    _, K, N = synth.LM_HEAD
    base = torch.from_numpy(synth.ternary_ptq(N // 16, K, seed=7)).to(dev)
    src = base.repeat(16, 1).contiguous()
    mats = [btf.repack_panels(src, N, K) for _ in range(2)]
    torch.cuda.synchronize()
    del src, base
    peak, peak_src = measured_peaks()
    nb = btf.gemv_max_nb(K)
    out = {"shape": f"K{K}_N{N}", "panel_bytes": btf.panel_bytes(N, K), "peak": peak, "peak_source": peak_src}
    st = torch.cuda.Stream(device=dev)

    def timed(launch):  # mean us per launch of a graph of `reps` launches (alternating weight copies)
        with torch.cuda.stream(st):
            for i in range(4):
                launch(mats[i % 2])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(reps):
                launch(mats[i % 2])
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        with torch.cuda.stream(st):
            g.replay()
        b.record(st)
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) * 1e3 / reps

    for M in (1, 8, 16):
        act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=8)).to(dev))
        y = torch.empty((M, N), device=dev)
        torch.cuda.synchronize()
        us = timed(lambda pm: btf.launch_gemv([(pm, y, N)], K, M, act, btf.STORE, st))
        gbs = synth.gemv_bytes(N, K, M) / us / 1e3
        out[f"M{M}"] = {"us": us, "GB/s": gbs, "frac_of_hbm": gbs / peak, "weight_passes": 1,
                        "bytes_per_launch": synth.gemv_bytes(N, K, M),
                        "path": "btf_gemv -> " + ("gemv_kernel" if M <= nb else "gemv_mma_kernel (warp int8 MMA)")}
        if M >= 9:  # the tcgen05 weight-major kernel on the same call, for comparison
            us_w = timed(lambda pm: btf.launch_gemm_wm([(pm, y, N)], K, M, act, btf.STORE, st))
            out[f"M{M}"]["weight_major"] = {"us": us_w, "GB/s": synth.gemv_bytes(N, K, M) / us_w / 1e3,
                                            "path": "btf_gemm_wm -> gemm_wm_kernel (tcgen05)"}
        if M > nb:  # the GEMV passes the MMA kernels replaced, on row views of the same activation
            def passes(pm):
                for m0 in range(0, M, nb):
                    sub = btf.Q8Act(act.q[m0:m0 + nb], act.d[m0:m0 + nb], act.s[m0:m0 + nb])
                    btf.launch_gemv([(pm, y[m0:m0 + nb], N)], K, min(nb, M - m0), sub, btf.STORE, st)
            us_p = timed(passes)
            out[f"M{M}"]["gemv_passes"] = {"us": us_p, "weight_passes": -(-M // nb),
                                           "GB/s": synth.gemv_bytes(N, K, M) / us_p / 1e3}
    out["device_error_word"] = btf.device_error()
    del mats
    return out


def load_config3(args):
    """Load path of benchmark configuration 3 (GGUF -> resident panels).

    Writes the 64-layer qwen35 GGUF with seeded weights (synth.write_qwen35_gguf),
    then times the memory plan (host only) and opening the decoder twice from
    the file: mmap, pinned staging, the GPU repack of every matrix into panels,
    and the step buffers. The first open reads the just-written file from the
    page cache. Each open then drops the file's pages (drop_page_cache), so on
    a disk-backed directory the second open reads the disk; on tmpfs both
    read memory. One decode step checks the loaded model, and the decoder's
    allocation total is checked against the plan."""
    import shutil

    import torch

    import btf_b200 as btf

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    btf.kernels_init(0)
    dims = dict(CONFIG3, n_layer=args.layers)
    tensors = synth.qwen35_tensors(dims)
    ptq = sum(ne[0] // 128 * 28 * ne[1] for _, ne, t in tensors if t == 143)
    need = ptq + sum(4 * int(np.prod(ne)) for _, ne, t in tensors if t != 143)
    dirs = [d for d in (os.environ.get("TMPDIR"), "/dev/shm", "/tmp", ROOT) if d and os.path.isdir(d)]
    room = [d for d in dirs if shutil.disk_usage(d).free > need * 1.25]
    if not room:
        raise SystemExit(f"no directory with {need * 1.25 / 1e9:.1f} GB free among {dirs}")
    path = os.path.join(room[0], f"btf_config3_{os.getpid()}.gguf")
    try:
        t0 = time.perf_counter()
        size = synth.write_qwen35_gguf(path, dims, seed=3)
        t_write = time.perf_counter() - t0
        t0 = time.perf_counter()
        plan = btf.plan_memory(path, n_ctx=4096)
        t_plan = time.perf_counter() - t0
        opens, first, held = [], None, None
        for i in range(2):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            dec = btf.Decoder(path, n_ctx=4096)
            torch.cuda.synchronize()
            opens.append(time.perf_counter() - t0)
            if i == 0:
                nxt, lg = dec.step(1, logits=True)
                first = (int(nxt), bool(np.all(np.isfinite(lg))))
                held = dec.info()["device_bytes"]
            dec.close()
    finally:
        os.remove(path)
    fs = ""
    try:
        fs = next((ln.split()[2] for ln in open("/proc/mounts") if ln.split()[1] == room[0]), "")
    except OSError:
        pass
    print(json.dumps({"load": "config3", "n_layer": dims["n_layer"], "dir": room[0], "fs": fs, "gguf_bytes": size,
                      "ptq1_0_bytes": ptq, "panel_bytes": plan["panel_bytes"], "write_s": round(t_write, 3),
                      "plan_s": round(t_plan, 4), "open_s": [round(t, 3) for t in opens],
                      "GB/s_ptq1_0": round(ptq / min(opens) / 1e9, 2), "device_bytes": held,
                      "device_bytes_planned": plan["device_bytes"], "staging_bytes": plan["staging_bytes"],
                      "first_step": {"token": first[0], "finite": first[1]}}))


def only_kernel(args):
    """Runs ONE config-1 GEMV kind (no graph) `--iters` times over 4 rotating weight
    copies (> L2), for profiler captures of a single kernel; prints per-launch us."""
    import torch

    import btf_b200 as btf

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    btf.kernels_init(0)
    if args.only == "decode":  # eager config-3 decode steps (one launch per kernel, no graph)
        with btf.Decoder(dims=CONFIG3, seed=3, n_ctx=4096, cuda_graph=False) as dec:
            t = 1
            for _ in range(args.iters):
                t, _ = dec.step(t)
            torch.cuda.synchronize()
            print(f"decode: {args.iters} eager steps, last token {t}, device error {btf.device_error()}")
        return
    if args.only in ("lmhead16", "lmhead16wm"):  # config 4's lm_head, batch 16: btf_gemv (routed to
        # btf_gemv_mma), or the tcgen05 weight-major kernel called directly
        _, K, N = synth.LM_HEAD
        M = 16
        base = torch.from_numpy(synth.ternary_ptq(N // 16, K, seed=7)).to(dev)
        src = base.repeat(16, 1).contiguous()
        mats = [btf.repack_panels(src, N, K) for _ in range(2)]
        del src, base
        act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=8)).to(dev))
        y = torch.empty((M, N), device=dev)
        launch = btf.launch_gemm_wm if args.only == "lmhead16wm" else btf.launch_gemv
        for i in range(args.iters):
            launch([(mats[i % 2], y, N)], K, M, act, btf.STORE)
        torch.cuda.synchronize()
        print(json.dumps({"kernel": args.only, "iters": args.iters, "device_error": btf.device_error()}))
        return
    if args.only == "gemm":  # one prefill GEMM: M=512, K=5120 -> N=17408
        M, K, N = 512, 5120, 17408
        src = torch.from_numpy(synth.ternary_ptq(N, K, seed=0)).to(dev)
        mats = [btf.repack_panels(src, N, K) for _ in range(2)]
        act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=2)).to(dev))
        y = torch.empty((M, N), device=dev)
        for i in range(args.iters):
            btf.launch_gemm([(mats[i % 2], y, N)], K, M, act, btf.STORE)
        torch.cuda.synchronize()
        print(json.dumps({"kernel": "gemm", "iters": args.iters, "device_error": btf.device_error()}))
        return
    K, segs_n, mode = {"qkv": (5120, ("q", "k", "v"), btf.STORE), "o": (6144, ("o",), btf.ADD),
                       "gateup": (5120, ("gate", "up"), btf.SWIGLU), "down": (17408, ("down",), btf.ADD)}[args.only]
    shapes = {n: N for n, _, N in synth.LAYER_SHAPES}
    srcs = {n: torch.from_numpy(synth.ternary_ptq(shapes[n], K, seed=0)).to(dev) for n in segs_n}
    copies = [{n: btf.repack_panels(srcs[n], shapes[n], K) for n in segs_n} for _ in range(4)]
    x = torch.from_numpy(synth.activations(1, K, seed=2)).to(dev)
    act = btf.quant_q8(x)
    ys = {n: torch.zeros((1, shapes[n]), device=dev) for n in segs_n}
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.iters)]
    for i in range(args.iters):
        c = copies[i % 4]
        segs = [(c[n], ys[n], shapes[n]) for n in segs_n]
        if mode == btf.SWIGLU:
            segs[1] = (c["up"], None, 0)
        ev[2 * i].record()
        if args.fused:
            btf.launch_gemv_f32(segs, K, 1, x, mode)
        else:
            btf.launch_gemv(segs, K, 1, act, mode)
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    us = [ev[2 * i].elapsed_time(ev[2 * i + 1]) * 1e3 for i in range(args.iters)]
    nbytes = sum(btf.panel_bytes(shapes[n], K) for n in segs_n)
    print(json.dumps({"kernel": args.only, "fused": bool(args.fused), "us": us,
                      "GB/s_weights_min_us": nbytes / min(us) / 1e3}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["qkv", "o", "gateup", "down", "gemm", "lmhead16", "lmhead16wm", "decode",
                                       "load"],
                    help="profile mode: one kernel kind, (lmhead16) config 4's lm_head at batch 16 through "
                         "btf_gemv (the warp-MMA GEMM), (lmhead16wm) the same on the weight-major tcgen05 GEMM, "
                         "(decode) eager config-3 decode steps, or (load) config 3 from a GGUF file into panels")
    ap.add_argument("--layers", type=int, default=64, help="--only load: layers of the config-3 model")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--fused", type=int, default=0, help="--only: 1 = btf_gemv_f32 (quantise inside the GEMV)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only == "load":
        load_config3(args)
    elif args.only:
        only_kernel(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
