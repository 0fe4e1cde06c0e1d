"""Benchmark of the B200 triangle-attention path (BASELINE.json metric: tri-attn ms/layer & TFLOP/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2|4|1|0]

One step = the starting-node layer then the ending-node layer (the pair a pairformer block runs,
pairformer.py:86-87), each with its residual add, on one batch of synthetic pair tensors:
    z1 = z + TriAttStart(z);  z2 = z1 + TriAttEnd(z1)
value = whole-job TFLOP/s with inputs resident in HBM (FLOPs per layer: 4 N^3 H C + 2 N^2 128 516 +
2 N^2 128 128, the reference's convention, tools/prof/triatt_common.py:51).  e2e = the same metric through
the C ABI with the pair tensor and mask copied host->device and the result device->host every step.

--impl reference: the reference's CPU path (the fp32 restatement in oracle/, run on the host cores
with all threads) on a bounded sample of attention rows of the same workload, extrapolated per layer.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, C, CZ, NPROJ = 4, 32, 128, 516
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CONFIGS = {
    0: dict(N=128, dtype="fp32", z_scale=1.0, pad="none", seed_z=0, seed_w=0, pair=False),
    1: dict(N=384, dtype="fp16", z_scale=1.0, pad="fixed38", seed_z=1, seed_w=1, pair=True),
    2: dict(N=1024, dtype="bf16", z_scale=0.5, pad="uniform15", seed_z=2, seed_w=2, pair=True),
    # 64 pairformer-style blocks of start+end triangle attention = 128 layers, distinct weights per layer
    3: dict(N=768, dtype="fp16", z_scale=1.0, pad="none", seed_z=3, seed_w=3, pair=True, blocks=64),
    4: dict(N=2048, dtype="bf16", z_scale=1.0, pad="frac05", seed_z=4, seed_w=4, pair=True),
}


def layer_flops(N: int, B: int = 1) -> dict:
    core = 4 * B * N ** 3 * H * C
    proj = 2 * B * N * N * CZ * NPROJ
    out = 2 * B * N * N * CZ * H * C
    return {"core": core, "proj": proj, "out": out, "total": core + proj + out}


# ---- synthetic inputs (same recipe as the test oracle's make_inputs) ------------------------------
def token_mask(N, pad, seed):
    t = torch.ones(N)
    if pad == "fixed38":
        t[N - 38:] = 0
    elif pad == "uniform15":
        g = torch.Generator().manual_seed(10_000 + seed)
        n_pad = int(torch.randint(0, int(0.15 * N) + 1, (1,), generator=g))
        if n_pad:
            t[N - n_pad:] = 0
    elif pad == "frac05":
        t[N - int(round(0.05 * N)):] = 0
    return t


def make_params(seed, gate_bias=1.0):
    g = torch.Generator().manual_seed(seed)
    std = (1.0 / CZ) ** 0.5
    shapes = {"w_q": (128, 128), "w_k": (128, 128), "w_v": (128, 128), "w_g": (128, 128), "w_b": (4, 128),
              "w_o": (128, 128)}
    p = {k: torch.randn(s, generator=g) * std for k, s in shapes.items()}
    p["ln_w"], p["ln_b"] = torch.ones(CZ), torch.zeros(CZ)
    p["g_b"] = torch.full((128,), float(gate_bias))
    return p


def make_config_inputs(cfg_id: int, N: int | None = None, B: int = 1):
    c = CONFIGS[cfg_id]
    N = c["N"] if N is None else N
    g = torch.Generator().manual_seed(c["seed_z"])
    z = torch.randn((B, N, N, CZ), generator=g) * c["z_scale"]
    t = token_mask(N, c["pad"], c["seed_z"])
    pm = (t[:, None] * t[None, :]).expand(B, N, N).contiguous()
    return z, pm, make_params(c["seed_w"]), make_params(c["seed_w"] + 100)


def stack_params(cfg_id: int, n_layers: int) -> list:
    """Distinct seeded weights for every layer of a stack (layer l: starting node when l is even)."""
    return [make_params(1000 * CONFIGS[cfg_id]["seed_w"] + l) for l in range(n_layers)]


class LayerStack:
    """A stack of start/end triangle-attention layers with residual adds, run in place on a device z
    through the C ABI (triattn_forward with add_residual=1), in one precision."""

    def __init__(self, N: int, params: list, precision: str, device):
        from boltz_mlx_b200 import _lib
        from boltz_mlx_b200.triangle_attention import TriangleAttention, load_params

        self.L, self.N, self.dt = _lib.lib(), N, _lib.dtype_code(precision)
        self.packs = []
        for l, p in enumerate(params):
            m = TriangleAttention(starting=(l % 2 == 0), precision=precision).to(device)
            load_params(m, {k: (v.to(device) if v is not None else None) for k, v in p.items()})
            self.packs.append(m.packed_weights(self.dt))
        self.wsb = _lib.workspace_bytes(1, N, N, self.dt)
        self.work = torch.empty(self.wsb, dtype=torch.uint8, device=device)

    def run(self, z, mask, stream):
        from boltz_mlx_b200 import _lib

        for l, pk in enumerate(self.packs):
            _lib.check(self.L.triattn_forward(z.data_ptr(), mask.data_ptr(), pk.data_ptr(), 1, self.N, int(l % 2 == 0),
                                              1e9, self.dt, 1, z.data_ptr(), self.work.data_ptr(), self.wsb, stream))


def stack_drift(cfg_id: int = 3, N: int | None = None, blocks: int | None = None, steps: int = 3,
                warmup: int = 1) -> dict:
    """Config 3: the 16-bit stack timed (sustained ms per layer) and its final z compared with the same
    stack run through the library's fp32 path (max_rel = max|d| / max|ref|, mean_abs, cos, and the same
    on the accumulated update z_final - z_0)."""
    from boltz_mlx_b200 import _lib

    c = CONFIGS[cfg_id]
    N = c["N"] if N is None else N
    n_layers = 2 * (c["blocks"] if blocks is None else blocks)
    dev = torch.device("cuda", torch.cuda.current_device())
    z0, pm, _, _ = make_config_inputs(cfg_id, N=N)
    z0, pm = z0.to(dev), pm.to(dev)
    params = stack_params(cfg_id, n_layers)
    stream = torch.cuda.current_stream(dev)
    s16 = LayerStack(N, params, c["dtype"], dev)
    z = z0.clone()
    for _ in range(warmup):
        z.copy_(z0)
        s16.run(z, pm, stream.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = 0.0
    for _ in range(steps):
        z.copy_(z0)
        e0.record(stream)
        s16.run(z, pm, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms += e0.elapsed_time(e1)
    ms_layer = ms / steps / n_layers
    z16 = z.clone()
    del s16
    s32 = LayerStack(N, params, "fp32", dev)
    z.copy_(z0)
    s32.run(z, pm, stream.cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device status word set"
    z32 = z

    def met(a, b):
        d = (a - b).double()
        bb = b.double()
        cos = float((a.double() * bb).sum() / (a.double().norm() * bb.norm()))
        return {"max_rel": float(d.abs().max() / bb.abs().max()), "mean_abs": float(d.abs().mean()), "cos": cos}

    out = {"N": N, "layers": n_layers, "precision": c["dtype"], "ms_per_layer": ms_layer,
           "z": met(z16, z32), "update": met(z16 - z0, z32 - z0),
           "ref_abs_max": float(z32.abs().max()), "update_abs_mean": float((z32 - z0).abs().mean())}
    return out


# ---- clocks -------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples every 50 ms around the timed region (median SM clock, throttle reasons): the
    timed region starts once the first sample has arrived (taken right after the warm-up, at load
    clocks), so even a short region carries a record."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx, self.rows, self.proc = gpu_index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 3.0:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return FALLBACK_PEAKS, "fallback"


# ---- distributed plumbing -------------------------------------------------------------------------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---- CPU reference / baseline -----------------------------------------------------------------------
_CPU_INPUTS: dict = {}


def cpu_sample_seconds(cfg_id: int, rows: int, threads: int) -> tuple[float, int]:
    """Seconds the CPU oracle (fp32, torch on the host cores) takes for `rows` attention rows of every
    layer of the step (both layers of a pair), including each layer's fixed part (LN + tri bias of all
    rows).  The config's inputs are generated once and reused."""
    from oracle.triattn_ref import tri_attention_ref  # CPU baseline leg only

    torch.set_num_threads(threads)
    if cfg_id not in _CPU_INPUTS:
        _CPU_INPUTS[cfg_id] = make_config_inputs(cfg_id)
    z, pm, ps, pe = _CPU_INPUTS[cfg_id]
    t0 = time.perf_counter()
    tri_attention_ref(z, pm, ps, starting=True, rows=(0, rows))
    if CONFIGS[cfg_id]["pair"]:
        tri_attention_ref(z, pm, pe, starting=False, rows=(0, rows))
    return time.perf_counter() - t0, z.shape[1]


def cpu_pair_seconds(cfg_id: int, threads: int, budget_s: float = 12.0) -> tuple[float, str]:
    """Per-pair CPU time, extrapolated from two bounded row samples (t = fixed + rows * per_row)."""
    t1, N = cpu_sample_seconds(cfg_id, 1, threads)
    r2 = max(2, min(N, int(budget_s / max(t1, 1e-3))))
    t2, _ = cpu_sample_seconds(cfg_id, r2, threads)
    per_row = max((t2 - t1) / (r2 - 1), 1e-9)
    fixed = max(t1 - per_row, 0.0)
    pair = fixed + per_row * N
    return pair, f"{r2} of {N} attention rows per layer (start+end), fixed LN/tri-bias part timed, extrapolated"


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    N = cfg["N"]
    threads = os.cpu_count() or 1
    fl = layer_flops(N)["total"] * (2 if cfg["pair"] else 1)
    torch.set_num_threads(threads)
    # Each step times a bounded sample: `rows` attention rows of both layers, which also pays each
    # layer's fixed part (LayerNorm + tri bias of ALL rows).  The pair time is then the same two-point
    # model as the cpu_baseline leg of the B200 arm, t = fixed + rows * per_row, with the one-row sample
    # giving the fixed part; the fixed part is counted once per layer, not N / rows times.
    t_one, _ = cpu_sample_seconds(args.config, 1, threads)
    rows = max(2, min(N, int(6.0 / max(t_one, 1e-3))))
    times, ones = [], [t_one]
    for i in range(args.warmup + args.steps):
        dt, _ = cpu_sample_seconds(args.config, rows, threads)
        if i >= args.warmup:
            times.append(dt)
            if len(ones) < 3:
                ones.append(cpu_sample_seconds(args.config, 1, threads)[0])
    t_rows, t1 = statistics.median(times), statistics.median(ones)
    per_row = max((t_rows - t1) / (rows - 1), 1e-9)
    fixed = max(t1 - per_row, 0.0)
    pair_s = fixed + per_row * N
    value = fl / pair_s / 1e12
    line = {
        "impl": "reference", "metric": metric_name(args.config), "value": value, "unit": "TFLOP/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": pair_s * 1e3,
        "ms_per_layer": pair_s * 1e3 / (2 if cfg["pair"] else 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.config, ws),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {N} attention rows per layer and step (and 1-row samples for the "
                                   f"fixed LN / tri-bias part), fitted as fixed + rows * per_row to the full pair",
                         "fixed_ms_per_pair": fixed * 1e3, "per_row_ms": per_row * 1e3},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def metric_name(cfg_id):
    N = CONFIGS[cfg_id]["N"]
    return f"tri-attn TFLOP/s, start+end pair, N={N}, B=1 (ms/layer reported beside it)"


def workload_config(cfg_id, ws):
    c = CONFIGS[cfg_id]
    return {"workload": f"config{cfg_id}: {'start+end pair' if c['pair'] else 'start node'} triangle attention, "
                        f"N={c['N']}, c_z=128, 4x32 heads, {c['dtype']}, B=1",
            "N": c["N"], "B": 1, "layers_per_step": 2 if c["pair"] else 1,
            "l2": "pair tensor (N^2 x 512 B) larger than the 126 MB L2 at N>=512; no flush",
            "parallelism": f"rows{ws}" if ws > 1 else "single"}


# ---- B200 arm --------------------------------------------------------------------------------------
def time_pair_one_gpu(cfg_id: int, dev, steps: int, warmup: int, precision=None) -> dict:
    """One configuration's start+end pair on one GPU through triattn_forward, inputs resident in HBM:
    ms per step (CUDA events over `steps` pairs after `warmup`) and the attention core alone."""
    from boltz_mlx_b200 import _lib
    from boltz_mlx_b200.triangle_attention import TriangleAttention, load_params

    cfg = CONFIGS[cfg_id]
    N = cfg["N"]
    prec = precision or cfg["dtype"]
    dt = _lib.dtype_code(prec)
    z_h, pm_h, ps, pe = make_config_inputs(cfg_id)
    packs = []
    for starting, p in ((True, ps), (False, pe)):
        m = TriangleAttention(starting=starting, precision=prec).to(dev)
        load_params(m, {k: (v.to(dev) if v is not None else None) for k, v in p.items()})
        packs.append(m.packed_weights(dt))
    z, mask = z_h.to(dev), pm_h.to(dev)
    t1, t2 = torch.empty_like(z), torch.empty_like(z)
    wsb = _lib.workspace_bytes(1, N, N, dt)
    work = torch.empty(wsb, dtype=torch.uint8, device=dev)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def step():
        _lib.check(L.triattn_forward(z.data_ptr(), mask.data_ptr(), packs[0].data_ptr(), 1, N, 1, 1e9, dt, 1,
                                     t1.data_ptr(), work.data_ptr(), wsb, sh))
        _lib.check(L.triattn_forward(t1.data_ptr(), mask.data_ptr(), packs[1].data_ptr(), 1, N, 0, 1e9, dt, 1,
                                     t2.data_ptr(), work.data_ptr(), wsb, sh))

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    step_ms = e0.elapsed_time(e1) / steps
    for _ in range(2):
        _lib.check(L.triattn_core(1, N, 0, N, dt, work.data_ptr(), wsb, sh))
    e0.record(stream)
    for _ in range(5):
        _lib.check(L.triattn_core(1, N, 0, N, dt, work.data_ptr(), wsb, sh))
    e1.record(stream)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device status word set"
    fl = layer_flops(N)
    core_ms = e0.elapsed_time(e1) / 5
    return {"metric": metric_name(cfg_id), "config": workload_config(cfg_id, 1), "precision": prec,
            "ms_per_step": step_ms, "ms_per_layer": step_ms / 2, "tflops": 2 * fl["total"] / (step_ms * 1e-3) / 1e12,
            "core_ms": core_ms, "core_tflops": fl["core"] / (core_ms * 1e-3) / 1e12, "steps": steps, "warmup": warmup}


def run_b200(args):
    from boltz_mlx_b200 import _lib
    from boltz_mlx_b200.triangle_attention import TriangleAttention, load_params

    ws_n, rank, local = dist_env()
    if ws_n > 1:
        from boltz_mlx_b200 import distributed as tdist

        return tdist.bench_sharded(args, make_config_inputs, layer_flops, workload_config, metric_name,
                                   ClockSampler, physical_gpu_index, peaks)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    N = cfg["N"]
    prec = args.precision or cfg["dtype"]
    dt = _lib.dtype_code(prec)
    z_h, pm_h, ps, pe = make_config_inputs(args.config)
    mods = []
    for starting, p in ((True, ps), (False, pe)):
        m = TriangleAttention(starting=starting, precision=prec).to(dev)
        load_params(m, {k: (v.to(dev) if v is not None else None) for k, v in p.items()})
        mods.append(m)
    packs = [m.packed_weights(dt) for m in mods]
    z = z_h.to(dev)
    mask = pm_h.to(dev)
    t1, t2 = torch.empty_like(z), torch.empty_like(z)
    wsb = _lib.workspace_bytes(1, N, N, dt)
    work = torch.empty(wsb, dtype=torch.uint8, device=dev)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    layers = (1 + int(cfg["pair"]))

    def step(src, mid, dst):
        _lib.check(L.triattn_forward(src.data_ptr(), mask.data_ptr(), packs[0].data_ptr(), 1, N, 1, 1e9, dt, 1,
                                     mid.data_ptr(), work.data_ptr(), wsb, sh))
        if cfg["pair"]:
            _lib.check(L.triattn_forward(mid.data_ptr(), mask.data_ptr(), packs[1].data_ptr(), 1, N, 0, 1e9, dt, 1,
                                         dst.data_ptr(), work.data_ptr(), wsb, sh))

    for _ in range(args.warmup):
        step(z, t1, t2)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device status word set during warm-up"

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu_index(local)) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step(z, t1, t2)
        ev1.record(stream)
        torch.cuda.synchronize()
    step_ms = ev0.elapsed_time(ev1) / args.steps
    fl = layer_flops(N)
    pair_flops = fl["total"] * layers
    value = pair_flops / (step_ms * 1e-3) / 1e12

    # ---- dominant kernel (attention core) timed alone, CUDA events on the launching stream ----
    _lib.check(L.triattn_mask_prep(mask.data_ptr(), 1, N, 0, 1e9, 0, N, dt, work.data_ptr(), wsb, sh))
    _lib.check(L.triattn_ln_proj(t1.data_ptr(), packs[1].data_ptr(), 1, N, 0, 0, N, dt, work.data_ptr(), wsb, sh))
    core_iters = 10
    for _ in range(2):
        _lib.check(L.triattn_core(1, N, 0, N, dt, work.data_ptr(), wsb, sh))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(core_iters):
        _lib.check(L.triattn_core(1, N, 0, N, dt, work.data_ptr(), wsb, sh))
    e1.record(stream)
    torch.cuda.synchronize()
    core_ms = e0.elapsed_time(e1) / core_iters
    # the two HBM-bound stages timed alone the same way (start-node views; out_proj writes t2, which the
    # e2e section below overwrites)
    def time_launch(fn, iters=10):
        for _ in range(2):
            fn()
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters
    stage_ms = {
        f"ln_proj_{nd}": time_launch(lambda st_=st_: _lib.check(L.triattn_ln_proj(
            t1.data_ptr(), packs[1].data_ptr(), 1, N, st_, 0, N, dt, work.data_ptr(), wsb, sh)))
        for nd, st_ in (("start", 1), ("end", 0))
    }
    stage_ms.update({
        f"out_proj_{nd}": time_launch(lambda st_=st_: _lib.check(L.triattn_out_proj(
            t1.data_ptr(), packs[1].data_ptr(), 1, N, st_, 0, N, dt, 1, t2.data_ptr(), work.data_ptr(), wsb, sh)))
        for nd, st_ in (("start", 1), ("end", 0))
    })
    hbm = peaks()[0].get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    stage_bytes = {"ln_proj": 1544 * N * N, "out_proj": 1536 * N * N}  # algorithmic bytes per launch
    stages = {k: {"ms": v, "frac_hbm": stage_bytes[k.rsplit("_", 1)[0]] / (v * 1e-3) / 1e9 / hbm}
              for k, v in stage_ms.items()}
    pk, pk_kind = peaks()
    tensor_peak = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    achieved = fl["core"] / (core_ms * 1e-3) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "core_traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(str(N))
        except ValueError:
            traffic = None

    # ---- e2e through the C ABI: host pinned buffers, every step's copies inside the timed region.
    #      As a serving loop would, steps are pipelined over two device slots: the input copy of step k
    #      (copy stream), the pair on the compute stream and the output copy (second copy stream) of
    #      step k - 1 overlap (PCIe is full duplex); events order each slot's copy -> compute -> copy ----
    zh = z_h.pin_memory()
    mh = pm_h.pin_memory()
    ohs = [torch.empty_like(zh).pin_memory() for _ in range(2)]
    zds = [torch.empty_like(z) for _ in range(2)]
    mds = [torch.empty_like(mask) for _ in range(2)]
    mids = [t1, torch.empty_like(z)]
    outs = [t2, torch.empty_like(z)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    ev_in = [ev(), ev()]
    ev_comp = [ev(), ev()]
    ev_out = [ev(), ev()]
    for e_ in ev_comp + ev_out:
        e_.record(stream)

    def e2e_step(k):
        s_ = k % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[s_])  # the slot's previous pair has read its inputs
            zds[s_].copy_(zh, non_blocking=True)
            mds[s_].copy_(mh, non_blocking=True)
            ev_in[s_].record(s_in)
        stream.wait_event(ev_in[s_])
        stream.wait_event(ev_out[s_])  # the slot's previous output has left the device
        _lib.check(L.triattn_forward(zds[s_].data_ptr(), mds[s_].data_ptr(), packs[0].data_ptr(), 1, N, 1, 1e9, dt, 1,
                                     mids[s_].data_ptr(), work.data_ptr(), wsb, sh))
        last = mids[s_]
        if cfg["pair"]:
            _lib.check(L.triattn_forward(mids[s_].data_ptr(), mds[s_].data_ptr(), packs[1].data_ptr(), 1, N, 0, 1e9, dt,
                                         1, outs[s_].data_ptr(), work.data_ptr(), wsb, sh))
            last = outs[s_]
        ev_comp[s_].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[s_])
            ohs[s_].copy_(last, non_blocking=True)
            ev_out[s_].record(s_out)

    # the timed window runs from the first step's input copy to the last step's output copy, so it holds
    # one pipeline fill (a pair and an output copy) on top of the steps: enough steps (2 x --steps, at
    # least 10) keep that share small; the steady-state period between consecutive output copies is
    # reported beside it
    e2e_steps = min(max(10, 2 * args.steps), 40)
    for k in range(2):
        e2e_step(k)
    torch.cuda.synchronize()
    t0, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    done = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    t0.record(s_in)
    for k in range(e2e_steps):
        e2e_step(k)
        done[k].record(s_out)
    t1e.record(s_out)
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1e) / e2e_steps
    e2e_steady_ms = done[2].elapsed_time(done[-1]) / (e2e_steps - 3)
    assert _lib.device_status() == 0, "device status word set"
    # every step computes the same pair: both slots' host copies must agree bit for bit
    assert torch.equal(ohs[0], ohs[1]), "pipelined e2e slots disagree"
    oh = ohs[0]

    # ---- config 4 (N=2048), where the north star's scaling target is quoted: the same pair on this GPU ----
    nested = cfg1 = None
    if args.config == 2:
        nested = time_pair_one_gpu(4, dev, args.steps, args.warmup, args.precision)
        # config 1 (N=384, fp16, the reference's CPU-runnable case) in its own precision; its 75 MB pair
        # tensor stays in L2 between steps, so this record is informational, not a bench value
        cfg1 = time_pair_one_gpu(1, dev, args.steps, args.warmup, None)
        cfg1["l2"] = "pair tensor (75 MB) fits in the 126 MB L2; no flush: informational"

    # ---- CPU baseline (oracle on the host cores, bounded sample) ----
    threads = os.cpu_count() or 1
    cpu_pair_s, sample = cpu_pair_seconds(args.config, threads, budget_s=args.cpu_budget)

    line = {
        "metric": metric_name(args.config), "value": value, "unit": "TFLOP/s", "n_gpus": 1,
        "gpu": torch.cuda.get_device_name(dev), "host_cores": os.cpu_count(),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "ms_per_layer": step_ms / layers,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": prec,
        "data": "synthetic: z~N(0,1)*scale, seeded trailing-padding pair mask, seeded N(0,1/128) weights",
        "config": workload_config(args.config, 1),
        "roofline": {"bound": "tensor", "kernel": "core_tc (flash attention core)", "achieved": achieved,
                     "peak": tensor_peak, "unit": "TFLOP/s", "frac": achieved / tensor_peak,
                     "peak_kind": f"{pk_kind} bf16 burst", "traffic": traffic, "core_ms": core_ms,
                     "algorithmic": f"F_core = 4 N^3 H C = {fl['core']:.4g} FLOP per launch"},
        "cpu_baseline": {"value": pair_flops / cpu_pair_s / 1e12, "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample, "ms_per_layer": cpu_pair_s * 1e3 / layers},
        "e2e": {"value": pair_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": zh.numel() * 4 + mh.numel() * 4, "d2h_bytes_per_step": oh.numel() * 4,
                "pipelined": "input copy, pair and output copy of consecutive steps overlap (2 device slots)",
                "steps": e2e_steps, "ms_per_step_steady": e2e_steady_ms,
                "window": "first input copy to last output copy (one pipeline fill included); "
                          "ms_per_step_steady = period between consecutive output copies after the fill"},
        "gpu_launches": args.steps * layers * 4,
        "clocks": clk.summary(),
        "stages": {**stages, "note": "HBM-bound stages timed alone with CUDA events (10 launches); frac_hbm = "
                   "algorithmic bytes (ln_proj 1544 B, out_proj 1536 B per pair) / time / measured copy peak"},
    }
    for key, rec in (("config4_same_gpus", nested), ("config1_same_gpus", cfg1)):
        if rec is not None:
            rec["core_frac"] = rec["core_tflops"] / tensor_peak
            line[key] = rec
    print(json.dumps(line), flush=True)


def trimul_flops(N: int, B: int = 1) -> dict:
    """Triangle multiplication per layer: the per-channel contraction 2 N^3 D, the projections
    2 N^2 D (4D + D) (p_in | g_in | g_out) and 2 N^2 D D (p_out)."""
    contraction = 2 * B * N ** 3 * CZ
    proj = 2 * B * N * N * CZ * (5 * CZ) + 2 * B * N * N * CZ * CZ
    return {"contraction": contraction, "proj": proj, "total": contraction + proj}


def run_trimul(args):
    """--layer trimul: one step = TriangleMultiplicationOutgoing then Incoming, each with its residual
    (the pairformer block's order), on the config's synthetic pair tensor and mask."""
    from boltz_mlx_b200 import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing, _lib, load_trimul_params

    def tm_params(seed):  # linears ~ N(0, 1/128), LayerNorm affine near identity
        g = torch.Generator().manual_seed(seed)
        p = {k: torch.randn(2 * CZ, CZ, generator=g) / CZ ** 0.5 for k in ("p_in", "g_in")}
        p.update({k: torch.randn(CZ, CZ, generator=g) / CZ ** 0.5 for k in ("p_out", "g_out")})
        for k in ("in", "out"):
            p[f"{k}_w"] = 1.0 + 0.1 * torch.randn(CZ, generator=g)
            p[f"{k}_b"] = 0.1 * torch.randn(CZ, generator=g)
        return p

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    N = args.case or cfg["N"]  # --case N: the same pair at a smaller N (ncu captures of a small case)
    prec = args.precision or cfg["dtype"]
    z_h, pm_h, _, _ = make_config_inputs(args.config, N=N)
    mods = [load_trimul_params(cls(128, precision=prec).to(dev), tm_params(cfg["seed_w"] + 50 + i))
            for i, cls in enumerate((TriangleMultiplicationOutgoing, TriangleMultiplicationIncoming))]
    z, mask = z_h.to(dev), pm_h.to(dev)
    t1, t2 = torch.empty_like(z), torch.empty_like(z)

    def step():
        torch.add(z, 0, out=t1)  # every step starts from the same input (the layers update in place)
        mods[0].forward_residual(t1, mask, inplace=True)
        mods[1].forward_residual(t1, mask, inplace=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu_index(0)) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    # the input copy (one N^2 x 512 B device copy per step) timed alone and taken out
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for _ in range(args.steps):
        torch.add(z, 0, out=t2)
    c1.record(stream)
    torch.cuda.synchronize()
    step_ms = (ev0.elapsed_time(ev1) - c0.elapsed_time(c1)) / args.steps
    fl = trimul_flops(N)
    line = {
        "metric": f"tri-mult TFLOP/s, outgoing+incoming pair, N={N}, B=1", "layer": "trimul",
        "value": 2 * fl["total"] / (step_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1,
        "gpu": torch.cuda.get_device_name(dev), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "ms_per_layer": step_ms / 2, "higher_is_better": True,
        "dtype": prec, "data": "synthetic: the config's pair tensor and mask, seeded N(0,1/128) weights",
        "config": {"workload": f"config{args.config}: tri-mult outgoing + incoming, N={N}, c_z=128, {prec}",
                   "N": N, "flops_per_layer": fl, "note": "input copy per step timed separately and subtracted"},
        "device_status": _lib.device_status(), "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_stack(args):
    """Config 3 line: sustained ms per layer of the 128-layer 16-bit stack and its drift against the
    same stack through the fp32 path."""
    torch.cuda.set_device(0)
    r = stack_drift(args.config, steps=args.steps, warmup=args.warmup)
    fl = layer_flops(r["N"])["total"]
    line = {"metric": f"tri-attn ms/layer, {r['layers']}-layer start+end stack, N={r['N']}, {r['precision']} (config 3)",
            "value": r["ms_per_layer"], "unit": "ms/layer", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "tflops": fl / (r["ms_per_layer"] * 1e-3) / 1e12, "dtype": r["precision"],
            "data": "synthetic: z~N(0,1), mask ones, distinct seeded N(0,1/128) weights per layer",
            "config": {"workload": f"config3: {r['layers']} layers, residual adds, N={r['N']}", "N": r["N"]},
            "drift_vs_fp32_path": {"z": r["z"], "update": r["update"]}}
    print(json.dumps(line), flush=True)


def run_case(args):
    """One start+end pair at N = args.case (bf16 unless --precision), for ncu captures of a small case."""
    from boltz_mlx_b200 import _lib
    from boltz_mlx_b200.triangle_attention import TriangleAttention, load_params

    dev = torch.device("cuda", 0)
    prec = args.precision or "bf16"
    z, pm, ps, pe = make_config_inputs(2, N=args.case)
    x, m = z.to(dev), pm.to(dev)
    mods = []
    for starting, p in ((True, ps), (False, pe)):
        mod = TriangleAttention(starting=starting, precision=prec).to(dev)
        load_params(mod, {k: (v.to(dev) if v is not None else None) for k, v in p.items()})
        mods.append(mod)
    for _ in range(2):
        y = x.clone()
        for mod in mods:
            y = mod.forward_residual(y, m, inplace=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device status word set"
    print(json.dumps({"case": args.case, "precision": prec, "mean_abs": float(y.abs().mean())}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=None)
    ap.add_argument("--precision", default=None)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="multi-GPU block exchange: peer stores from the output projection + cross-GPU barrier "
                         "(default), or NCCL all-to-alls")
    ap.add_argument("--layer", default="triattn", choices=["triattn", "trimul"],
                    help="triattn: the north-star start+end pair (default); trimul: triangle multiplication "
                         "outgoing + incoming on the same config (single GPU)")
    ap.add_argument("--case", type=int, default=None,
                    help="profiling case: run one start+end pair at this N once (after one warm-up pair), "
                         "check the device status and exit; nothing is timed")
    args = ap.parse_args()
    if args.config is None:
        args.config = 2  # one workload for every GPU count, so the driver's scaling ratios compare like with like
    if args.layer == "trimul":
        run_trimul(args)
        return
    if args.case is not None:
        run_case(args)
        return
    if args.layer == "trimul":
        run_trimul(args)
    elif args.impl == "b200" and "blocks" in CONFIGS[args.config]:
        run_stack(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
