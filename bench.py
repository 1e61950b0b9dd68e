"""Benchmark of the HiF4 W4A4 Linear hot path on B200.

A step is one pass of the Qwen3-8B-shaped W4A4 linear set at T = 8192 prefill
tokens: for each of q/k/v/o/gate/up/down, K1 (HiSQ1024 rotation + three-level
HiF4 activation quantization) then K3 (tcgen05 GEMM against HiF4 weights).
``value`` is whole-job TFLOPS (2*T*N*K summed over the projections and ranks)
with inputs resident in HBM; ``e2e`` is the same metric through the public
module API (``FakeQuantLinear``) with pinned host inputs copied in and outputs
copied out every step. The attention hot path (causal GQA
32/8 heads, S = 32768) is measured in the same run and reported under
``attention``.

``--impl reference`` times the reference's own CPU path on the host instead: its
``FakeQuantLinear`` in CPU torch on all host threads when the reference is importable
(an offline install under ``baseline/_ref``), else ``oracle/linear_torch.py``, a CPU-torch
restatement with the same bits and cost; a step is 1024 of the 8192 tokens through all
seven projections.

Launch: ``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 under
``torch.distributed.run`` (one process per GPU, replicas: the linear set does not
shard, so every rank runs its own copy and no collective is on the data path).

The same line carries the two sharded workloads, strong scaling over the N ranks:
``wan22_block`` (the Wan2.2 DiT block, attention sharded by heads,
row-parallel o / ffn.2 with an NCCL all-reduce) and ``qwen3_32b_prefill`` (config 5:
the 64-layer Qwen3-32B prefill, tensor-parallel with two NCCL all-reduces per layer).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT / "faquant-public_b200"), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "W4A4 GEMM & HiF4 QK/PV attn TFLOPS (% of B200 peak); prefill tokens/s"
T_TOKENS = 8192
PROJECTIONS = [  # (reference module path, in_features, out_features) -- Qwen3-8B
    ("self_attn.q_proj", 4096, 4096),
    ("self_attn.k_proj", 4096, 1024),
    ("self_attn.v_proj", 4096, 1024),
    ("self_attn.o_proj", 4096, 4096),
    ("mlp.gate_proj", 4096, 12288),
    ("mlp.up_proj", 4096, 12288),
    ("mlp.down_proj", 12288, 4096),
]
ATT = dict(batch=1, hq=32, hkv=8, seq=32768, d=128)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def linear_flops(tokens: int = T_TOKENS, out_frac: float = 1.0) -> float:
    return sum(2.0 * tokens * k * int(n * out_frac) for _, k, n in PROJECTIONS)


def bench_config(world: int) -> dict:
    """The workload both arms report (the reference arm times a bounded sample of it)."""
    return {"workload": "qwen3-8b W4A4 linear set, T=8192 (BASELINE config 2)", "tokens": T_TOKENS,
            "projections": [p for p, _, _ in PROJECTIONS], "rotation": "hisq1024 (seed 17)",
            "levels": "123", "weights": "GPTQ HiF4 of N(0,0.02) (damp 0.01, group 64, block 128, H from "
            "the rotated step activations; the CPU arm's time does not depend on the weight values and "
            "it quantizes them by RTN)", "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (512 MB activations + 436 MB weights per step)"}


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ distributed
def gpu_numa_cpus(device) -> tuple[int, set[int]] | None:
    """The NUMA node the GPU's PCIe slot hangs off and that node's CPUs (from sysfs), or
    None where the box does not say. Pinned host buffers placed on that node keep the
    host <-> device copies off the socket interconnect."""
    import torch

    try:
        prop = torch.cuda.get_device_properties(device)
        bus = f"{getattr(prop, 'pci_domain_id', 0):04x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus: set[int] = set()
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        return (node, cpus) if cpus else None
    except (AssertionError, AttributeError, OSError, RuntimeError, ValueError):
        return None


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def init_dist(world: int, backend: str):
    import datetime

    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":  # one GPU per rank, named, so NCCL does not guess the mapping
            import torch

            # NCCL's communicator lines (rank, nranks, transport) in the log, as evidence of
            # the ranks the collectives ran on
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"

            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    return dist if world > 1 else None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ GPU workload
def _rotated_fp32(x, signs, perm, block: int):
    """The reader rotation in fp32 (``x * signs``, gather, block Hadamard, ``/sqrt(block)``)
    by a Hadamard matrix product: GPTQ's calibration input, where the last bits of the
    Hessian do not matter."""
    import torch

    h = torch.ones(1, 1, device=x.device)
    while h.shape[0] < block:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    r = (x.float() * signs.float())[:, perm]
    return (r.view(r.shape[0], -1, block) @ h).view_as(r) / float(block) ** 0.5


def gptq_weight(w, x_rot):
    """GPTQ with HiF4 grids (this library's GPU solver, ``faquant_b200.gptq``) at the deployed
    settings -- damp 0.01, groups of 64, block 128 -- with the Hessian from the rotated
    activations. Returns the bf16 grid weight and its packed form (metadata from the solver)."""
    import torch

    from faquant_b200 import ops
    from faquant_b200.gptq import GPTQ

    n, k = w.shape
    lin = torch.nn.Linear(k, n, bias=False, device=w.device, dtype=torch.float32)
    with torch.no_grad():
        lin.weight.copy_(w.float())
    gp = GPTQ(lin)
    gp.add_batch(x_rot)
    gp.quantize(quant_format="hif4", bits=4, group_size=64, damp=0.01, block_size=128,
                capture_hif4_metadata=True)
    meta = lin.faquant_hif4_qat_parameters
    wq = lin.weight.detach().to(torch.bfloat16)
    wc, wm, bad = ops.hif4_pack_weight(wq, scale=meta.scale.reshape(n, k // 64),
                                       lv2=meta.scale_lv2_exponent.reshape(n, k // 64, 8),
                                       lv3=meta.scale_lv3_exponent.reshape(n, k // 64, 16))
    if bad:
        raise RuntimeError(f"GPTQ weight does not pack onto its own metadata ({bad} values)")
    del gp, lin
    return wq, wc, wm


def build_linear_set(device, seed: int = 0, weights: str = "gptq"):
    """Config 2's seven projections: activations N(0,1) with 0.5 % outlier channels x20 (bf16),
    weights N(0,0.02) quantized onto the HiF4 grid by GPTQ (``weights="gptq"``, Hessian from
    the step's own rotated activations, as the configuration states) or by RTN."""
    import torch

    from faquant_b200 import ops
    from faquant_b200.hisq_rotation import derive_hisq_rotation

    g = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for path, k, n in PROJECTIONS:
        x = torch.randn(T_TOKENS, k, device=device, generator=g)
        outliers = torch.randperm(k, device=device, generator=g)[: max(1, round(0.005 * k))]
        x[:, outliers] *= 20.0
        x = x.to(torch.bfloat16)
        w = (torch.randn(n, k, device=device, generator=g) * 0.02).to(torch.bfloat16)
        rot = derive_hisq_rotation(f"model.layers.0.{path}", k, seed=17, block_size=1024)
        signs, perm = rot.signs.to(device), rot.permutation.to(device)
        if weights == "gptq":
            wq, wc, wm = gptq_weight(w, _rotated_fp32(x, signs, perm, 1024))
        else:
            wq, _, _ = ops.hif4_quantize(w, levels="123")  # RTN onto the HiF4 grid
            wc, wm, _ = ops.hif4_pack_weight(w, levels="123")  # the same grid, 4.5-bit packed
        layers.append(dict(path=path, k=k, n=n, x=x, w=wq, wc=wc, wm=wm, signs=signs, perm=perm,
                           y=torch.empty(T_TOKENS, n, device=device, dtype=torch.bfloat16)))
        del w
        torch.cuda.empty_cache()
    return layers


def run_linear_step(layers, timers=None):
    from faquant_b200 import ops

    launches = 0
    for L in layers:
        if timers is not None:
            timers["q0"].append(timers["ev"]())
        xq, _, _ = ops.hif4_quantize(L["x"], levels="123", signs=L["signs"], permutation=L["perm"], rot_block=1024)
        if timers is not None:
            timers["g0"].append(timers["ev"]())
        ops.gemm_bf16(xq, L["w"], out=L["y"])
        if timers is not None:
            timers["g1"].append(timers["ev"]())
        launches += 2
    return launches


def run_packed_step(layers, timers=None, kernel=False):
    """The same step with the weights held packed, as FakeQuantLinear(packed_weights=True)
    runs it: from PACKED_EXPAND_MIN_ROWS input rows (by default every call) K1 writes the bf16
    QDQ, the weight is expanded to bf16 (faq_hif4_dequantize) and K3 runs; with `kernel`
    (or fewer rows) K1 writes the activation's codes and the W4A4 GEMM expands both
    operands tile by tile (faq_w4a4_gemm)."""
    from faquant_b200 import ops
    from faquant_b200.quantization import PACKED_EXPAND_MIN_ROWS

    launches = 0
    for L in layers:
        if not kernel and L["x"].shape[0] >= PACKED_EXPAND_MIN_ROWS:
            launches += 3
            xq, _, _ = ops.hif4_quantize(L["x"], levels="123", signs=L["signs"], permutation=L["perm"],
                                         rot_block=1024)
            if timers is not None:
                timers["x0"].append(timers["ev"]())
            w = ops.hif4_dequantize(L["wc"], L["wm"], L["k"])
            if timers is not None:
                timers["g0"].append(timers["ev"]())
            ops.gemm_bf16(xq, w, out=L["y"])
        else:
            launches += 2
            _, codes, meta = ops.hif4_quantize(L["x"], levels="123", signs=L["signs"], permutation=L["perm"],
                                               rot_block=1024, want_qdq=False, want_codes=True)
            if timers is not None:
                timers["x0"].append(timers["ev"]())
                timers["g0"].append(timers["x0"][-1])
            ops.w4a4_gemm((codes, meta), L["wc"], L["wm"], out=L["y"])
        if timers is not None:
            timers["g1"].append(timers["ev"]())
    return launches


def run_decode_linear(layers, device, pk):
    """The config-2 projections at decode sizes (1 and 16 rows): FakeQuantLinear modules with
    bf16 weights (K1 + K3) against the same modules holding packed weights (K1 + the
    small-row kernel, faq_w4a4_gemm_qdq_a), the seven calls of a step captured in one CUDA
    graph as a decode loop captures them (host work out of the timing). Weight bytes bound
    these calls: 386 MB of bf16 weights against 109 MB packed per step."""
    import torch

    from faquant_b200.quantization import FakeQuantLinear

    kw = dict(quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64, symmetric=True,
              clip_ratio=1.0, quantize_weight=False, input_rotation_block_size=1024)
    plain, packed = [], []
    for L in layers:
        lin = torch.nn.Linear(L["k"], L["n"], bias=False, device="meta")
        lin.weight = torch.nn.Parameter(L["w"], requires_grad=False)
        rot = dict(input_rotation_signs=L["signs"], input_rotation_permutation=L["perm"])
        plain.append(FakeQuantLinear(lin, **kw, **rot))
        pm = FakeQuantLinear(lin, **kw, **rot, packed_weights=False)
        pm.use_packed(L["wc"], L["wm"])
        packed.append(pm)
    w_bf16 = sum(2 * L["w"].numel() for L in layers)
    w_packed = sum(L["wc"].numel() + 4 * L["wm"].numel() for L in layers)

    def graph_us(mods, xs, reps=20):
        s = torch.cuda.Stream(device=device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(s):
            for _ in range(2):
                for m, x in zip(mods, xs):
                    m(x)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        # thread_local: under torchrun the process group's watchdog thread queries its
        # events while this thread captures; only this thread's calls must be capturable
        with torch.no_grad(), torch.cuda.graph(g, capture_error_mode="thread_local"):
            for _ in range(reps):
                for m, x in zip(mods, xs):
                    m(x)
        g.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) * 1000 / reps
            best = us if best is None else min(best, us)
        del g
        return best

    out = {"workload": "the seven config-2 projections per decode step, FakeQuantLinear, CUDA-graph replay",
           "weight_bytes_bf16": w_bf16, "weight_bytes_packed": w_packed}
    for rows in (1, 16):
        xs = [L["x"][:rows].contiguous() for L in layers]
        us_b = graph_us(plain, xs)
        us_p = graph_us(packed, xs)
        out[f"rows_{rows}"] = {
            "bf16_weights_us_per_step": us_b, "packed_us_per_step": us_p, "speedup": us_b / us_p,
            "packed_weight_gbs": w_packed / (us_p * 1e-6) / 1e9,
            "packed_frac_of_hbm": w_packed / (us_p * 1e-6) / 1e9 / pk["hbm_gbs"],
            "bf16_weight_gbs": w_bf16 / (us_b * 1e-6) / 1e9,
        }
    return out


def build_attention(device, seed: int = 1):
    import torch

    b, hq, hkv, s, d = ATT["batch"], ATT["hq"], ATT["hkv"], ATT["seq"], ATT["d"]
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(b, hq, s, d, device=device, generator=g).to(torch.bfloat16)
    k = torch.randn(b, hkv, s, d, device=device, generator=g).to(torch.bfloat16)
    v = torch.randn(b, hkv, s, d, device=device, generator=g).to(torch.bfloat16)
    lo, hi = math.log(0.5), math.log(2.0)
    smooth = torch.exp(torch.rand(d, device=device, generator=g) * (hi - lo) + lo)
    return dict(q=q, k=k, v=v, smooth=smooth, out=torch.empty(b, s, hq, d, device=device, dtype=torch.bfloat16))


def run_attention_step(A, timers=None):
    from faquant_b200 import ops

    qd, _, _ = ops.qk_prep(A["q"], levels="123", rotate=True, smooth_scale=A["smooth"], smooth_mode="mul")
    kd, _, _ = ops.qk_prep(A["k"], levels="123", rotate=True, smooth_scale=A["smooth"], smooth_mode="div")
    vd, _, _ = ops.qk_prep(A["v"], levels="123", rotate=False)
    if timers is not None:
        timers["a0"].append(timers["ev"]())
    ops.hif4_attention(qd, kd, vd, causal=True, p_levels="123", quantized_normalizer=True, out=A["out"])
    if timers is not None:
        timers["a1"].append(timers["ev"]())
    return 4


def attention_e2e(A, args, device, barrier, dist):
    """Config-3 attention through the public calls a model makes, from pinned host buffers:
    Q/K/V go up (one side stream, the next step's while this one computes), the model-side
    transform of qwen3._attention_forward (faq_qk_prep: Smooth-QK and the Hadamard, one bf16
    cast) and the HF attention backend (simulated_flash_attention_forward: Q/K/V HiF4, then
    K5), the output comes down on another stream. Every byte crosses PCIe inside the timed
    region; time on the device, max over ranks."""
    import torch

    from faquant_b200 import ops
    from faquant_b200.attention import new_simulated_attention_stats, simulated_flash_attention_forward

    module = torch.nn.Module()
    module.is_causal = True
    module.faquant_attention_query_chunk_size = 128
    module.faquant_attention_key_chunk_size = 128
    module.faquant_qk_matmul_quant = True
    module.faquant_pv_matmul_quant = True
    module.faquant_pv_normalizer_mode = "quantized_same"
    module.faquant_matmul_quant_kwargs = {"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                          "clip_ratio": 1.0}
    module.faquant_simulated_attention_stats = new_simulated_attention_stats()
    host = {n: A[n].cpu().pin_memory() for n in ("q", "k", "v")}
    out_shape = A["out"].shape
    host_out = torch.empty(out_shape, dtype=torch.bfloat16).pin_memory()
    host_out.zero_()
    main = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)

    def upload():
        with torch.cuda.stream(s_in):
            dev_in = {n: host[n].to(device, non_blocking=True) for n in host}
            ev = torch.cuda.Event()
            ev.record(s_in)
        return dev_in, ev

    def step(dev_in, ev):
        main.wait_event(ev)
        for t in dev_in.values():
            t.record_stream(main)
        qh = ops.qk_prep(dev_in["q"], levels=None, rotate=True, smooth_scale=A["smooth"], smooth_mode="mul")[0]
        kh = ops.qk_prep(dev_in["k"], levels=None, rotate=True, smooth_scale=A["smooth"], smooth_mode="div")[0]
        out, _ = simulated_flash_attention_forward(module, qh, kh, dev_in["v"], None, scaling=128**-0.5)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            host_out.copy_(out, non_blocking=True)
        out.record_stream(s_out)

    nxt = upload()
    for _ in range(2):
        cur, nxt = nxt, upload()
        step(*cur)
    torch.cuda.synchronize()
    steps = max(2, args.att_steps)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    nxt = upload()
    for i in range(steps):
        cur = nxt
        if i + 1 < steps:
            nxt = upload()
        step(*cur)
    main.wait_stream(s_out)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = torch.tensor([e0.elapsed_time(e1) / steps], device=device)
    if dist is not None:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    world = dist.get_world_size() if dist is not None else 1
    return {"value": attention_flops() * world / (float(e_ms.item()) * 1e-3) / 1e12, "unit": "TFLOPS",
            "ms_per_step": float(e_ms.item()),
            "h2d_bytes_per_step": sum(h.numel() * 2 for h in host.values()),
            "d2h_bytes_per_step": host_out.numel() * 2,
            "path": "pinned host Q/K/V -> faq_qk_prep (model transform) -> simulated_flash_attention_forward "
                    "(HF backend: Q/K/V HiF4 + K5) -> pinned host output"}


def attention_flops() -> float:
    s = ATT["seq"]
    return 4.0 * ATT["d"] * ATT["hq"] * ATT["batch"] * s * (s + 1) / 2.0


def flush_l2(buf):
    buf.add_(1.0)


# ------------------------------------------------------------------ CPU legs (reference path)
REF_DIR = ROOT / "baseline" / "_ref"


def _import_reference():
    """The reference's own modules from an offline install under baseline/_ref, or None."""
    if not (REF_DIR / "faquant").is_dir():
        return None
    sys.path.insert(0, str(REF_DIR))
    try:
        import faquant.hisq_rotation as hr
        import faquant.quantization as q
    except Exception:  # noqa: BLE001 - an unusable install falls back to the port
        return None
    return hr, q


def cpu_linear_set(tokens: int, seed: int = 0):
    """The seven config-2 projections on `tokens` rows (full K and N) as CPU forwards.

    With the reference importable, each forward is the reference's own
    ``FakeQuantLinear`` (src/faquant/quantization.py:199-277) built as its module does
    (RTN weight at construction, not timed); otherwise the CPU-torch restatement
    ``oracle/linear_torch.py``, which gives the same bits and, measured against the
    reference on 8 cores, 0.93-1.09x its time. Returns (kind, [(x, forward)]).
    """
    import torch

    from oracle import linear_torch as lt

    ref = _import_reference()
    g = torch.Generator().manual_seed(seed)
    out = []
    for path, k, n in PROJECTIONS:
        x = torch.randn(tokens, k, generator=g)
        x[:, torch.randperm(k, generator=g)[: max(1, round(0.005 * k))]] *= 20.0
        x = x.to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        name = f"model.layers.0.{path}"
        if ref is not None:
            hr, q = ref
            rot = hr.derive_hisq_rotation(name, k, seed=17, block_size=1024)
            lin = torch.nn.Linear(k, n, bias=False).to(torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(w)
            mod = q.FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                                    symmetric=True, clip_ratio=1.0, input_rotation_signs=rot.signs,
                                    input_rotation_permutation=rot.permutation, input_rotation_block_size=1024)
            out.append((x, mod))
        else:
            from faquant_b200.hisq_rotation import derive_hisq_rotation

            rot = derive_hisq_rotation(name, k, seed=17, block_size=1024)
            wq = lt.hif4_fake_quantize(w, "123")

            def fwd(xx, wq=wq, rot=rot):
                return lt.fake_quant_linear(xx, wq, None, levels="123", signs=rot.signs, permutation=rot.permutation,
                                            block=1024)

            out.append((x, fwd))
        del w
    return ("reference" if ref is not None else "port"), out


def cpu_linear_step(linears) -> None:
    import torch

    with torch.no_grad():
        for x, fwd in linears:
            fwd(x)


def cpu_threads() -> int:
    import torch

    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def cpu_sample_text(kind: str, tokens: int, threads: int, steps: int, warmup: int) -> str:
    what = ("the reference's own FakeQuantLinear (src/faquant/quantization.py:199-277, imported from "
            "baseline/_ref)" if kind == "reference" else
            "oracle/linear_torch.py, the CPU-torch restatement of the reference's FakeQuantLinear (same bits; "
            "0.93-1.09x the reference's time on 8 cores)")
    return (f"{tokens} of the 8192 tokens through all 7 projections (full K and N): HiSQ1024 rotation, three-level "
            f"HiF4 and the bf16 F.linear of {what}, CPU torch on {threads} threads, {steps} steps after {warmup} "
            f"warm-up")


def cpu_baseline(tokens: int = 1024, steps: int = 2) -> dict:
    threads = cpu_threads()
    kind, linears = cpu_linear_set(tokens)
    cpu_linear_step(linears)  # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_linear_step(linears)
    dt = (time.perf_counter() - t0) / steps
    return {
        "value": linear_flops(tokens) / dt / 1e12, "unit": "TFLOPS", "cores": threads, "kind": kind,
        "sample": cpu_sample_text(kind, tokens, threads, steps, 1), "seconds_per_step": dt,
    }


def cpu_attention_baseline(seq: int = ATT["seq"], heads: int = 1) -> dict:
    """The reference's own attention simulator (``simulated_flash_attention_forward``,
    src/faquant/simulated_flash_attention.py:457-909, imported from baseline/_ref) with config
    3's settings -- causal, HiF4 Q/K/V and P in groups of 64, P-Reordering
    (``quantized_same``), query chunks of 256 and key chunks of 128 -- on the host cores: a
    bounded sample of ``heads`` query heads (with their KV head) at the full sequence length;
    its work per (query, key) pair is that of the full configuration, 32 heads."""
    import torch

    if _import_reference() is None:
        return {"unavailable": "the reference is not importable (no offline install under baseline/_ref)"}
    from types import SimpleNamespace

    from faquant.simulated_flash_attention import new_simulated_attention_stats, simulated_flash_attention_forward

    threads = cpu_threads()
    d = ATT["d"]

    def module():
        return SimpleNamespace(
            is_causal=True, training=False, faquant_attention_query_chunk_size=256,
            faquant_attention_key_chunk_size=128, faquant_qk_matmul_quant=True, faquant_pv_matmul_quant=True,
            faquant_pv_normalizer_mode="quantized_same",
            faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                         "clip_ratio": 1.0},
            faquant_simulated_attention_stats=new_simulated_attention_stats())

    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, heads if i == 0 else 1, seq, d, generator=g).to(torch.bfloat16) for i in range(3))
    with torch.no_grad():
        simulated_flash_attention_forward(module(), q[:, :, :1024], k[:, :, :1024], v[:, :, :1024], None,
                                          scaling=d ** -0.5)  # warm-up
        t0 = time.perf_counter()
        simulated_flash_attention_forward(module(), q, k, v, None, scaling=d ** -0.5)
        dt = time.perf_counter() - t0
    flops = 4.0 * d * heads * seq * (seq + 1) / 2.0
    return {"value": flops / dt / 1e12, "unit": "TFLOPS", "cores": threads, "kind": "reference",
            "sample": f"{heads} of the {ATT['hq']} query heads (with its KV head) at the full S={seq}, causal: the "
                      f"reference's simulated_flash_attention_forward (HiF4 Q/K/V and P, P-Reordering, query chunk "
                      f"256, key chunk 128), CPU torch on {threads} threads, one call after a 1024-token warm-up; "
                      f"the full configuration is {ATT['hq'] // heads}x this work",
            "seconds": dt, "seconds_full_config_estimate": dt * ATT["hq"] / heads}


def reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if world > 1 and rank != 0:
        return
    tokens = 1024
    threads = cpu_threads()
    kind, linears = cpu_linear_set(tokens)
    for _ in range(args.warmup):
        cpu_linear_step(linears)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_linear_step(linears)
    dt = (time.perf_counter() - t0) / args.steps
    value = linear_flops(tokens) / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": bench_config(world),
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": kind,
                         "sample": cpu_sample_text(kind, tokens, threads, args.steps, args.warmup)},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ main arm
def main_arm(args) -> None:
    import torch

    from faquant_b200 import _lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = init_dist(world, "nccl")
    _lib.load()
    pk, pk_kind = peaks()

    layers = build_linear_set(device, seed=rank)
    A = build_attention(device, seed=1000 + rank) if not args.no_attention else None
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    ev = lambda: (lambda e: (e.record(), e)[1])(torch.cuda.Event(enable_timing=True))  # noqa: E731
    # ---------------- device-resident timing of the linear set
    for _ in range(args.warmup):
        run_linear_step(layers)
    timers = {"q0": [], "g0": [], "g1": [], "ev": ev}
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        launches = 0
        for _ in range(args.steps):
            launches += run_linear_step(layers, timers)
        end.record()
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    gemm_ms = sum(a.elapsed_time(b) for a, b in zip(timers["g0"], timers["g1"]))
    quant_ms = sum(a.elapsed_time(b) for a, b in zip(timers["q0"], timers["g0"]))
    n_gemm = len(timers["g0"])
    ms_t = torch.tensor([ms], device=device)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = linear_flops() * world / (ms_max * 1e-3) / 1e12
    gemm_tflops = linear_flops() * args.steps / (gemm_ms * 1e-3) / 1e12
    quant_bytes = sum(T_TOKENS * k * (2 + 2) for _, k, _ in PROJECTIONS)  # bf16 read + bf16 QDQ write
    nproj = len(PROJECTIONS)
    per_proj = {
        p: {"quantize_ms": sum(timers["q0"][i].elapsed_time(timers["g0"][i]) for i in range(j, n_gemm, nproj))
            / args.steps,
            "gemm_ms": sum(timers["g0"][i].elapsed_time(timers["g1"][i]) for i in range(j, n_gemm, nproj))
            / args.steps}
        for j, (p, _, _) in enumerate(PROJECTIONS)
    }
    quant_gbs = quant_bytes * args.steps / (quant_ms * 1e-3) / 1e9

    # ---------------- the same step with packed weights (FakeQuantLinear(packed_weights=True))
    packed = None
    if not args.no_packed:
        def timed_packed(kernel):
            run_linear_step(layers)
            ref_out = [L["y"].clone() for L in layers]
            run_packed_step(layers, kernel=kernel)
            same = all(torch.equal(a.view(torch.int16), L["y"].view(torch.int16)) for a, L in zip(ref_out, layers))
            del ref_out
            for _ in range(args.warmup):
                run_packed_step(layers, kernel=kernel)
            ptimers = {"x0": [], "g0": [], "g1": [], "ev": ev}
            barrier()
            torch.cuda.synchronize()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record()
            for _ in range(args.steps):
                launches = run_packed_step(layers, ptimers, kernel=kernel)
            p1.record()
            torch.cuda.synchronize()
            barrier()
            p_ms = p0.elapsed_time(p1) / args.steps
            g_ms = sum(a.elapsed_time(b) for a, b in zip(ptimers["g0"], ptimers["g1"])) / args.steps
            x_ms = sum(a.elapsed_time(b) for a, b in zip(ptimers["x0"], ptimers["g0"])) / args.steps
            return p_ms, g_ms, x_ms, same, launches

        p_ms, p_gemm_ms, p_x_ms, same, launches = timed_packed(False)
        k_ms, k_gemm_ms, _, k_same, k_launches = timed_packed(True)
        w_vals = sum(L["wc"].numel() * 2 for L in layers)
        packed = {
            "workload": "the config-2 step with 4.5-bit packed weights as FakeQuantLinear(packed_weights=True) runs "
                        "it at 8192 rows: K1 bf16 QDQ, the weight expanded to bf16 (faq_hif4_dequantize), K3",
            "ms_per_step": p_ms, "tflops": linear_flops() / (p_ms * 1e-3) / 1e12,
            "expand_ms_per_step": p_x_ms,
            "expand_gbs": w_vals * (0.5625 + 2.0) / (p_x_ms * 1e-3) / 1e9 if p_x_ms > 0 else None,
            "gemm_ms_per_step": p_gemm_ms, "gemm_tflops": linear_flops() / (p_gemm_ms * 1e-3) / 1e12,
            "weight_bytes_packed": sum(L["wc"].numel() + 4 * L["wm"].numel() for L in layers),
            "weight_bytes_bf16": sum(2 * L["w"].numel() for L in layers),
            "bit_identical_to_bf16_path": same,
            "gpu_launches_per_step": launches,
            "packed_gemm_kernel": {
                "workload": "the same step on faq_w4a4_gemm (K1 writes codes, both operands expanded in shared "
                            "memory tile by tile; the module's path below PACKED_EXPAND_MIN_ROWS rows)",
                "ms_per_step": k_ms, "gemm_ms_per_step": k_gemm_ms,
                "gemm_tflops": linear_flops() / (k_gemm_ms * 1e-3) / 1e12,
                "gemm_frac_of_bf16_peak": linear_flops() / (k_gemm_ms * 1e-3) / 1e12 / pk["bf16_tflops"],
                "bit_identical_to_bf16_path": k_same, "gpu_launches_per_step": k_launches,
            },
        }

    # ---------------- the projections at decode sizes: packed weights streamed by the small-row kernel
    dec_lin = None
    if not args.no_packed:
        dec_lin = run_decode_linear(layers, device, pk)

    # ---------------- attention (config 3), device-resident
    att = None
    if A is not None:
        for _ in range(max(1, args.warmup // 3)):
            run_attention_step(A)
        atimers = {"a0": [], "a1": [], "ev": ev}
        a_steps = max(1, args.att_steps)
        barrier()
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(a_steps):
            launches_att = run_attention_step(A, atimers)
        s1.record()
        torch.cuda.synchronize()
        barrier()
        a_ms = s0.elapsed_time(s1) / a_steps
        k_ms = sum(a.elapsed_time(b) for a, b in zip(atimers["a0"], atimers["a1"])) / a_steps
        att = {
            "workload": "qwen3-8b causal GQA attention prefill (BASELINE config 3)", **ATT,
            "ms_per_step": a_ms, "kernel_ms": k_ms,
            "tflops": attention_flops() / (a_ms * 1e-3) / 1e12,
            "kernel_tflops": attention_flops() / (k_ms * 1e-3) / 1e12,
            "frac_of_bf16_peak": attention_flops() / (k_ms * 1e-3) / 1e12 / pk["bf16_tflops"],
            "tokens_per_s": ATT["seq"] * ATT["batch"] / (a_ms * 1e-3),
            "gpu_launches_per_step": launches_att,
        }

    # ---------------- the same attention end to end through the public API, host buffers
    if att is not None and not args.no_e2e:
        att["e2e"] = attention_e2e(A, args, device, barrier, dist)

    # ---------------- the reference's own GPU kernel beside K5 (config 4 attention), rank 0
    gpu_ref = None
    # one GPU's comparison; at N > 1 the other ranks would wait at the next barrier while
    # rank 0 compiles and runs the reference's Triton kernel
    if A is not None and world == 1 and not args.no_gpu_reference:
        gpu_ref = gpu_reference_attention(2)

    # ---------------- decode step (K6): one new token per sequence against a 32K-key cache
    dec = None
    if A is not None:
        dec = run_decode(args, device, pk, barrier, dist)

    # ---------------- sharded workloads (configs 4 and 5), strong scaling over the ranks
    tp_lines = {}
    if not args.no_tp:
        del layers, A
        torch.cuda.empty_cache()
        tp_lines = run_tp_workloads(args, rank, world, device, pk, barrier, dist)
        layers = build_linear_set(device, seed=rank) if not args.no_e2e else None

    # ---------------- e2e through FakeQuantLinear with host buffers
    e2e = None
    if not args.no_e2e:
        from faquant_b200.quantization import FakeQuantLinear

        mods, host_x, host_y = [], [], []
        # allocate (and so place) the pinned buffers from CPUs of the GPU's NUMA node
        numa = gpu_numa_cpus(device)
        saved_affinity = os.sched_getaffinity(0)
        if numa is not None:
            os.sched_setaffinity(0, numa[1])
        for L in layers:
            lin = torch.nn.Linear(L["k"], L["n"], bias=False, device="meta")
            lin.weight = torch.nn.Parameter(L["w"], requires_grad=False)
            m = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                                symmetric=True, clip_ratio=1.0, quantize_weight=False,
                                input_rotation_signs=L["signs"], input_rotation_permutation=L["perm"],
                                input_rotation_block_size=1024)
            mods.append(m)
            host_x.append(L["x"].cpu().pin_memory())
            host_y.append(torch.empty(T_TOKENS, L["n"], dtype=torch.bfloat16).pin_memory())
            host_y[-1].zero_()  # touch the pages here, on this node
        os.sched_setaffinity(0, saved_affinity)

        # The projections' host copies are pipelined with their compute, as a serving loop
        # streams batches: inputs go up on one side stream, outputs come down on another
        # (PCIe is full duplex, the copy engines are separate), the compute stream waits for
        # each input, and the next step's inputs go up while this step's outputs still come
        # down. Projections with the largest outputs go first, so the download starts early.
        # The timed region ends when the last output of the last step is on the host: every
        # byte of every step crosses PCIe inside it.
        main = torch.cuda.current_stream()
        s_in, s_out = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
        order = sorted(range(len(mods)), key=lambda i: -host_y[i].numel())

        def e2e_step():
            xs, ev_in = [], []
            with torch.cuda.stream(s_in):
                for i in order:
                    xs.append(host_x[i].to(device, non_blocking=True))
                    ev = torch.cuda.Event()
                    ev.record(s_in)
                    ev_in.append(ev)
            for i, x, ev in zip(order, xs, ev_in):
                main.wait_event(ev)
                x.record_stream(main)
                y = mods[i](x)
                done = torch.cuda.Event()
                done.record(main)
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    host_y[i].copy_(y, non_blocking=True)
                y.record_stream(s_out)

        for _ in range(2):
            e2e_step()
        e_steps = max(6, args.steps // 10)
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        s_in.wait_stream(main)  # no copy starts before e0
        s_out.wait_stream(main)
        for _ in range(e_steps):
            e2e_step()
        main.wait_stream(s_out)  # e1 follows the last output's arrival on the host
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e_ms = torch.tensor([e0.elapsed_time(e1) / e_steps], device=device)
        if dist is not None:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": linear_flops() * world / (float(e_ms.item()) * 1e-3) / 1e12, "unit": "TFLOPS",
               "ms_per_step": float(e_ms.item()),
               "h2d_bytes_per_step": sum(h.numel() * 2 for h in host_x),
               "d2h_bytes_per_step": sum(h.numel() * 2 for h in host_y),
               "host_numa_node": None if numa is None else numa[0]}

    if rank == 0:
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.exists():
            traffic = json.loads(tfile.read_text()).get("gemm_bytes_per_launch")
        avg_gemm_ms = gemm_ms / n_gemm
        gemm_flops_per_launch = linear_flops() / len(PROJECTIONS)
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": bench_config(world),
            "tokens_per_s": T_TOKENS * world / (ms_max * 1e-3),
            "roofline": {
                "kernel": "gemm_bf16_tn_pair_kernel", "bound": "tensor", "achieved": gemm_tflops,
                "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": gemm_tflops / pk["bf16_tflops"],
                "peak_kind": f"{pk_kind} bf16 burst", "traffic": traffic,
                "avg_launch_ms": avg_gemm_ms, "algorithmic_flops_per_launch_avg": gemm_flops_per_launch,
                "frac_of_sustained_peak": gemm_tflops / pk.get("bf16_tflops_sustained", pk["bf16_tflops"]),
                "frac_of_fp8_dense_nominal": gemm_tflops / 4500.0,
                "frac_of_fp4_dense_nominal": gemm_tflops / 9000.0,
            },
            "quantize_kernel": {"kernel": "hif4_rotate_v4_kernel", "bound": "hbm", "achieved": quant_gbs,
                                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": quant_gbs / pk["hbm_gbs"],
                                "ms_per_step": quant_ms / args.steps},
            "per_projection_ms": per_proj,
            "clocks": clocks.summary(),
            "gpu_launches": launches,
            "packed_linear_set": packed,
            "decode_linear_set": dec_lin,
            "attention": att,
            "gpu_reference": gpu_ref,
            "decode": dec,
            **tp_lines,
            "e2e": e2e,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
            if att is not None and world == 1:
                try:
                    att["cpu_baseline"] = cpu_attention_baseline()
                except Exception as exc:  # noqa: BLE001 - a reported baseline never costs the bench line
                    att["cpu_baseline"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _timed(fn, steps: int, warmup: int, barrier, dist, device) -> float:
    """Device time of ``fn`` per step in ms, max over ranks (barrier + synchronize around)."""
    import torch

    for _ in range(warmup):
        fn()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=device)
    if dist is not None:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def run_decode(args, device, pk: dict, barrier, dist) -> dict:
    """Config-3 shapes in decode: batch 1, 32 q / 8 kv heads, one new position against a
    cache of 32768 keys (HiF4 operands prepared once, as the append cache keeps them)."""
    import torch

    from faquant_b200 import ops

    b, hq, hkv, sk = 1, ATT["hq"], ATT["hkv"], ATT["seq"]
    g = torch.Generator(device=device).manual_seed(11)
    q = ops.qk_prep(torch.randn(b, hq, 1, 128, device=device, generator=g).to(torch.bfloat16), levels="123")[0]
    k = ops.qk_prep(torch.randn(b, hkv, sk, 128, device=device, generator=g).to(torch.bfloat16), levels="123")[0]
    v = ops.qk_prep(torch.randn(b, hkv, sk, 128, device=device, generator=g).to(torch.bfloat16), levels="123",
                    rotate=False)[0]
    ws = torch.empty(int(ops._lib.load().faq_hif4_decode_workspace_bytes(b, hq, hkv, 1, sk, 128)),
                     dtype=torch.uint8, device=device)
    out = torch.empty(b, 1, hq, 128, dtype=torch.bfloat16, device=device)
    ms = _timed(lambda: ops.hif4_decode_attention(q, k, v, out=out, workspace=ws), 20, 3, barrier, dist, device)
    kv_bytes = 2 * b * hkv * sk * 128 * 2
    return {"workload": "qwen3-8b decode step: 1 token, 32/8 heads, 32768-key HiF4 K/V cache (config-3 shapes)",
            "ms_per_step": ms, "tokens_per_s": b / (ms * 1e-3), "kv_bytes": kv_bytes,
            "achieved_gbs": kv_bytes / (ms * 1e-3) / 1e9, "frac_of_hbm_peak": kv_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
            "gpu_launches_per_step": 3, "steps": 20}


def _collective_share(tp, step, step_ms: float, world: int, barrier) -> dict | None:
    """One more step with the collectives (all-reduces; with sequence parallelism the
    reduce-scatters and all-gathers) timed by CUDA events on the streams they run on: their
    summed device time and bytes against the timed step (an untimed extra step, so the
    events cannot perturb the measurement above). Overlapped chunks (side stream) count in
    full, so `share` bounds the exposed communication from above. Bus bytes per rank: an
    all-reduce moves 2 (n - 1) / n of its tensor, a reduce-scatter or all-gather (n - 1) / n
    of the full tensor."""
    import torch

    if world == 1:
        return None
    tp.timer = []
    barrier()
    step()
    torch.cuda.synchronize()
    kinds = {}
    for a, b, n, kind in tp.timer:
        k = kinds.setdefault(kind, {"calls_per_step": 0, "bytes_per_step": 0, "ms_per_step": 0.0})
        k["calls_per_step"] += 1
        k["bytes_per_step"] += n
        k["ms_per_step"] += a.elapsed_time(b)
    tp.timer = None
    bus = 0.0
    for kind, k in kinds.items():
        f = 2 * (world - 1) / world if kind == "all_reduce" else (world - 1) / world
        bus += k["bytes_per_step"] * f
        k["bus_gbs"] = k["bytes_per_step"] * f / (k["ms_per_step"] * 1e-3) / 1e9 if k["ms_per_step"] > 0 else None
    ms = sum(k["ms_per_step"] for k in kinds.values())
    return {"calls_per_step": sum(k["calls_per_step"] for k in kinds.values()),
            "bytes_per_step": sum(k["bytes_per_step"] for k in kinds.values()), "bus_bytes_per_step": bus,
            "ms_per_step": ms, "share_of_step": ms / step_ms, "bus_gbs": bus / (ms * 1e-3) / 1e9 if ms > 0 else None,
            "by_kind": kinds,
            "collective": "NCCL over NVLink: all_reduce(sum, bf16) of row-parallel outputs, or with sequence "
                          "parallelism reduce_scatter(sum, bf16) of them and all_gather of the packed HiF4 codes "
                          "and meta (bf16 in the bf16 layers); all_gather of Wan's per-head sums of squares"}


def _e2e_timed(fn, host_in, steps: int, device, barrier, dist) -> dict:
    """A sharded workload end to end from pinned host memory: every step uploads its input
    (one side stream; the next step's while this one computes), runs `fn` on it through the
    workload's public module, and downloads the output on another stream; the timed region
    ends when the last output is on the host. Device time, max over ranks; bytes per rank."""
    import torch

    main = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    outs = {}

    def upload():
        with torch.cuda.stream(s_in):
            x = host_in.to(device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
        return x, ev

    def step(x, ev):
        main.wait_event(ev)
        x.record_stream(main)
        y = fn(x)
        if "host" not in outs:
            outs["host"] = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            outs["host"].copy_(y, non_blocking=True)
        y.record_stream(s_out)

    step(*upload())  # warm-up, allocates the pinned output
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    nxt = upload()
    for i in range(steps):
        cur = nxt
        if i + 1 < steps:
            nxt = upload()
        step(*cur)
    main.wait_stream(s_out)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = torch.tensor([e0.elapsed_time(e1) / steps], device=device)
    if dist is not None:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    out_bytes = outs["host"].numel() * outs["host"].element_size()
    del outs
    return {"ms_per_step": float(e_ms.item()), "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": out_bytes}


def run_tp_workloads(args, rank: int, world: int, device, pk: dict, barrier, dist) -> dict:
    """BASELINE configs 4 (Wan2.2 block, heads sharded) and 5 (Qwen3-32B TP prefill)."""
    import torch

    from faquant_b200.tensor_parallel import (Qwen3TPConfig, Qwen3TPPrefill, TPGroup, WanBlockConfig, WanBlockTP,
                                              default_input_ids)

    tp = TPGroup(rank, world, None)
    out = {}
    wcfg = WanBlockConfig()
    block = WanBlockTP(wcfg, tp, device)
    g = torch.Generator(device=device).manual_seed(7)
    x = torch.randn(wcfg.seq, wcfg.dim, generator=g, device=device).to(torch.bfloat16)
    lay = block.seq_layout(wcfg.seq)
    if lay is not None:  # sequence parallel: a block of a DiT takes and passes on its rank's token rows
        x = x[lay.owned(device)].contiguous()
        run_block = lambda: block.forward_shard(x, lay)  # noqa: E731
        w_io = f"this rank's {lay.shard_rows} token rows in and out (sequence parallel, {lay.chunks} chunks)"
    else:
        run_block = lambda: block(x)  # noqa: E731
        w_io = "all 75600 token rows in and out"
    w_ms = _timed(run_block, args.tp_steps, 1, barrier, dist, device)
    w_comm = _collective_share(tp, run_block, w_ms, world, barrier)
    wf = wcfg.flops()
    out["wan22_block"] = {
        "workload": "Wan2.2-A14B DiT block, S=75600 (21x45x80), 40 heads, self-attention + FFN (BASELINE config 4)",
        "parallelism": f"heads/tensor-parallel x{world}", "scaling": "strong", "ms_per_step": w_ms,
        "tflops": wf["total"] / (w_ms * 1e-3) / 1e12, "frac_of_bf16_peak":
        wf["total"] / (w_ms * 1e-3) / 1e12 / (pk["bf16_tflops"] * world),
        "tokens_per_s": wcfg.seq / (w_ms * 1e-3), "flops": wf, "steps": args.tp_steps,
        "rotation": "rbhn_r64 readers (column-parallel), signs r64 (row-parallel)", "levels": wcfg.levels,
        "io": w_io, "collectives": w_comm,
    }
    if not args.no_e2e:
        e2e = _e2e_timed((lambda xs: block.forward_shard(xs, lay)) if lay is not None else block,
                         x.cpu().pin_memory(), args.tp_steps, device, barrier, dist)
        e2e.update({"value": wf["total"] / (e2e["ms_per_step"] * 1e-3) / 1e12, "unit": "TFLOPS",
                    "path": ("pinned host token rows of this rank -> WanBlockTP.forward_shard (sequence "
                             "parallel) -> pinned host output rows of this rank") if lay is not None else
                            "pinned host hidden states -> WanBlockTP -> pinned host output"})
        out["wan22_block"]["e2e"] = e2e
    del block, x
    torch.cuda.empty_cache()
    qcfg = Qwen3TPConfig(layers=args.qwen_layers)
    model = Qwen3TPPrefill(qcfg, tp, device)
    ids = default_input_ids(4, 8192, qcfg.vocab, device)
    q_ms = _timed(lambda: model(ids), args.tp_steps, 1, barrier, dist, device)
    q_comm = _collective_share(tp, lambda: model(ids), q_ms, world, barrier)
    qf = qcfg.flops(4, 8192)
    q_e2e = None
    if not args.no_e2e:
        q_e2e = _e2e_timed(model, ids.cpu().pin_memory(), args.tp_steps, device, barrier, dist)
        q_e2e.update({"value": 4 * 8192 / (q_e2e["ms_per_step"] * 1e-3), "unit": "tokens/s",
                      "path": "pinned host token ids -> Qwen3TPPrefill -> pinned host logits"})
    out["qwen3_32b_prefill"] = {
        "workload": f"Qwen3-32B prefill, {qcfg.layers} layers, batch 4 x 8192 tokens (BASELINE config 5)",
        "parallelism": f"tensor-parallel x{world}", "scaling": "strong", "ms_per_forward": q_ms,
        "tokens_per_s": 4 * 8192 / (q_ms * 1e-3), "tflops": qf["total"] / (q_ms * 1e-3) / 1e12,
        "frac_of_bf16_peak": qf["total"] / (q_ms * 1e-3) / 1e12 / (pk["bf16_tflops"] * world),
        "flops": qf, "steps": args.tp_steps, "bf16_layers": list(qcfg.bf16_layers),
        "rotation": "hisq1024 per norm (column-parallel), signs r64 (row-parallel)",
        "logits": "last position of each sequence", "weights": "RTN HiF4 of N(0,0.02)",
        "collectives": q_comm, "e2e": q_e2e,
    }
    del model
    torch.cuda.empty_cache()
    return out


def kernel_case(name: str, reps: int) -> None:
    """One kernel on a profiling-sized case (inputs > L2, a few GB at most), for ncu."""
    import torch

    from faquant_b200 import ops
    from faquant_b200.hisq_rotation import derive_hisq_rotation

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if name == "gemm":  # q_proj-shaped: 8192 x 4096 x 4096 (A 64 MB + B 32 MB + Y 64 MB)
        a, _, _ = ops.hif4_quantize(torch.randn(8192, 4096, device=dev, generator=g).to(torch.bfloat16))
        b, _, _ = ops.hif4_quantize((torch.randn(4096, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16))
        y = torch.empty(8192, 4096, device=dev, dtype=torch.bfloat16)
        for _ in range(reps):
            ops.gemm_bf16(a, b, out=y)
    elif name == "quantize":  # gate_proj input: 8192 x 4096 bf16, HiSQ1024
        x = torch.randn(8192, 4096, device=dev, generator=g).to(torch.bfloat16)
        rot = derive_hisq_rotation("model.layers.0.mlp.gate_proj", 4096, seed=17, block_size=1024)
        s, p = rot.signs.to(dev), rot.permutation.to(dev)
        for _ in range(reps):
            ops.hif4_quantize(x, levels="123", signs=s, permutation=p, rot_block=1024)
    elif name == "attention":  # 8 q heads / 2 kv heads, S = 8192, causal
        q = torch.randn(1, 8, 8192, 128, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 2, 8192, 128, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 2, 8192, 128, device=dev, generator=g).to(torch.bfloat16)
        qd, _, _ = ops.qk_prep(q, levels="123", rotate=True)
        kd, _, _ = ops.qk_prep(k, levels="123", rotate=True)
        vd, _, _ = ops.qk_prep(v, levels="123", rotate=False)
        for _ in range(reps):
            ops.hif4_attention(qd, kd, vd, causal=True, p_levels="123", quantized_normalizer=True)
    elif name == "decode":  # one token, 32 q / 8 kv heads, 32768-key HiF4 cache (config-3 shapes)
        q = torch.randn(1, 32, 1, 128, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 8, 32768, 128, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 8, 32768, 128, device=dev, generator=g).to(torch.bfloat16)
        for _ in range(reps):
            ops.hif4_decode_attention(q, k, v)
    elif name == "w4a4":  # the packed GEMM, 2048 x 4096 x 4096: both operands packed, then A as bf16 QDQ
        x = torch.randn(2048, 4096, device=dev, generator=g).to(torch.bfloat16)
        xq, ac, am = ops.hif4_quantize(x, levels="123", want_codes=True)
        w = (torch.randn(4096, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        bc, bm, _ = ops.hif4_pack_weight(w, levels="123")
        for _ in range(reps):
            ops.w4a4_gemm((ac, am), bc, bm)
            ops.w4a4_gemm(xq, bc, bm)
    elif name == "decode_linear":  # K3s on down_proj at one row, then the bf16 expansion of the gate weight
        w = (torch.randn(4096, 12288, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        bc, bm, _ = ops.hif4_pack_weight(w, levels="123")
        a, _, _ = ops.hif4_quantize(torch.randn(1, 12288, device=dev, generator=g).to(torch.bfloat16), levels="123")
        for _ in range(reps):
            ops.w4a4_gemm(a, bc, bm)
        wg = (torch.randn(12288, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        gc, gm, _ = ops.hif4_pack_weight(wg, levels="123")
        for _ in range(reps):
            ops.hif4_dequantize(gc, gm, 4096)
    elif name == "wan_operands":  # K4 on a Wan qkv output: 16800 tokens x 40 heads (config-4 heads)
        from faquant_b200.tensor_parallel import rope3d_tables

        seq, heads, d = 16800, 40, 128
        n = heads * d
        qkv = torch.randn(seq, 3 * n, device=dev, generator=g).to(torch.bfloat16)
        cos, sin = rope3d_tables((21, 10, 80), d, 10000.0, dev)
        w = torch.ones(n, device=dev)
        view = lambda lo: qkv[:, lo:lo + n].view(1, seq, heads, d).transpose(1, 2)  # noqa: E731
        out = torch.empty(1, heads, seq, d, dtype=torch.bfloat16, device=dev)
        for _ in range(reps):
            head_ss = ops.row_sumsq(qkv[:, :2 * n], segments=2 * heads)[None]
            ops.wan_qk_prep(view(0), head_ss, w, cos=cos, sin=sin, out=out)
            ops.qk_prep(view(2 * n), rotate=False, out=out)
            ops.qk_prep(view(2 * n), rotate=True, out=out)
    else:
        raise SystemExit(f"unknown kernel case {name!r}")
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": name, "reps": reps, "ok": True}))


def gpu_reference_attention(reps: int) -> dict:
    """The reference's own GPU kernel -- its Triton HiF4 attention
    (`wan22_attention.hif4_attention`, src/faquant/wan22_attention.py:165-183) -- against K5
    on BASELINE config 4 (Wan2.2: 75 600 tokens, 40 heads, non-causal, HiF4 P,
    P-Reordering), the same HiF4-prepared operands for both, on this GPU. The reference is
    imported from an offline install under baseline/_ref; without it the block says
    `unavailable` and why."""
    import importlib

    import torch

    try:
        if not (REF_DIR / "faquant").is_dir():
            raise ImportError(f"no reference install under {REF_DIR.relative_to(ROOT)}")
        sys.path.insert(0, str(REF_DIR))
        ref = importlib.import_module("faquant.wan22_attention")
    except Exception as e:  # noqa: BLE001 - the install is optional
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    from faquant_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    seq, heads, d = 75600, 40, 128
    g = torch.Generator(device=dev).manual_seed(0)
    prep = [ops.qk_prep(torch.randn(1, heads, seq, d, device=dev, generator=g).to(torch.bfloat16), levels="123",
                        rotate=rot)[0] for rot in (True, True, False)]
    views = [t[0].transpose(0, 1) for t in prep]  # the reference's [L, H, D]

    def timed(fn):
        out = fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            out = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, out

    ms_ref, o_ref = timed(lambda: ref.hif4_attention(*views, softmax_scale=d**-0.5, quantize_p=True,
                                                     quantized_normalizer=True))
    ms_our, o_our = timed(lambda: ops.hif4_attention(*prep, scale=d**-0.5, causal=False, p_levels="123",
                                                     quantized_normalizer=True))
    flops = 4.0 * d * heads * seq * seq
    a, b = o_our[0].float(), o_ref.float()
    result = {"kernel": "triton hif4_attention (wan22_attention.py:165-183)",
              "workload": "BASELINE config 4 attention: 75600 tokens, 40 heads, d 128, non-causal",
              "reference_ms": ms_ref, "reference_tflops": flops / ms_ref / 1e9, "ours_ms": ms_our,
              "ours_tflops": flops / ms_our / 1e9, "speedup": ms_ref / ms_our,
              "rel_fro_diff": float((a - b).double().norm() / b.double().norm()),
              "values_differing": int((a != b).sum()), "values": a.numel(),
              "max_abs_diff": float((a - b).abs().max()), "reps": reps}
    del prep, views, o_ref, o_our, a, b
    torch.cuda.empty_cache()
    return result


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--att-steps", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-attention", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-packed", action="store_true", help="skip the packed-weight step")
    ap.add_argument("--no-gpu-reference", action="store_true",
                    help="skip timing the reference's Triton attention beside K5")
    ap.add_argument("--no-tp", action="store_true", help="skip the sharded workloads (configs 4 and 5)")
    ap.add_argument("--tp-steps", type=int, default=2)
    ap.add_argument("--qwen-layers", type=int, default=64)
    ap.add_argument("--kernel-case", choices=["gemm", "quantize", "attention", "decode", "wan_operands", "w4a4",
                                              "decode_linear"],
                    help="run one kernel on a profiling-sized case (for ncu) and exit")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--gpu-reference", action="store_true",
                    help="time the reference's Triton attention (baseline/_ref) beside K5 on config 4 and exit")
    args = ap.parse_args()
    if args.gpu_reference:
        print(json.dumps({"gpu_reference": gpu_reference_attention(args.reps)}))
        return
    if args.kernel_case:
        kernel_case(args.kernel_case, args.reps)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        main_arm(args)


if __name__ == "__main__":
    main()
