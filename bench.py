"""Benchmark: mask-aware attention TFLOP/s on B200, 1..8 GPUs.

Workload: non-softmax attention, B=32, H=32, S=8192,
D=128, bf16, non-causal -- sigmoid(QK^T/sqrt(D) - log S) V and
ReLU(QK^T/sqrt(D)) V / S. One step runs both operators over this rank's shard
of the B*H = 1024 independent (batch, head) units; the units are split
evenly across ranks (no collective on the data path), so total work is fixed
as N grows ("strong" scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

FLOPs are mask-aware: 4 * D * visible_pairs * units (masked pairs never
count). Timing: W warm-up steps, then K steps between a barrier +
synchronize on both sides, CUDA events on the launching stream, max over
ranks. Inputs (6.4 GB per GPU at N=1) exceed the 126 MB L2, so no flush is
needed between steps. Rank 0 prints one JSON line.

``--impl reference`` times the reference's eager CPU implementation (the
fp32 restatement in ``oracle/``, the reference's algorithm on the host cores,
all threads) on a bounded sample of the same workload and prints the same
JSON line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

B_TOTAL, H_TOTAL, S, D = 32, 32, 8192, 128
SPEC_BF16_TFLOPS = 2250.0
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "mask-aware attention TFLOP/s (sigmoid + ReLU, config 5)"
L2_BYTES = 126 * 1024 * 1024
SUITE_MIN_MS = 25.0    # shortest timed region of a suite entry
SUITE_MAX_ITERS = 400
HOST_CYCLES_PER_LAUNCH = 250_000  # device cycles of lead per queued launch (> host dispatch)


def device_lead(n_launches: int):
    """Queue a device-side wait long enough for the host to enqueue
    n_launches calls before the first of them runs, so that CUDA events
    around those calls measure device time rather than the Python dispatch
    of each call (which can exceed a short launch)."""
    if hasattr(torch.cuda, "_sleep"):
        torch.cuda._sleep(int(min(n_launches, SUITE_MAX_ITERS) * HOST_CYCLES_PER_LAUNCH))
# The workload both arms measure (printed as `config` by each).
CONFIG = {"workload": "config 5: sigmoid(s - log S) and ReLU(s)/S attention, non-causal",
          "B": B_TOTAL, "H": H_TOTAL, "S": S, "D": D}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {k: float(d[k]) for k in FALLBACK if k in d}, "measured"
    return dict(FALLBACK), "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def shard(units: int, ws: int, rank: int):
    """Contiguous, even split of ``units`` (batch*head pairs) over ``ws`` ranks."""
    lo = units * rank // ws
    hi = units * (rank + 1) // ws
    return lo, hi


def max_over_ranks(x: float, device, ws: int) -> float:
    """The largest ``x`` over all ranks (every rank gets it)."""
    t = torch.tensor([x], dtype=torch.float64, device=device)
    if ws > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_max(vals, device, ws: int):
    """Element-wise maximum of the list ``vals`` over all ranks."""
    e = torch.tensor(list(vals), dtype=torch.float64, device=device)
    if ws > 1:
        import torch.distributed as dist
        gathered = [torch.zeros_like(e) for _ in range(ws)]
        dist.all_gather(gathered, e)
        e = torch.stack(gathered).max(0).values
    return [float(x) for x in e]


def variants():
    import chia_proj_b200 as cp
    return [
        ("sigmoid_attn", lambda q, k, v: cp.sigmoid_attn(q, k, v, causal=False, bias=-math.log(S)),
         dict(causal=False, bias=-math.log(S))),
        ("relu_attn", lambda q, k, v: cp.relu_attn(q, k, v, causal=False, out_scale=1.0 / S),
         dict(causal=False, out_scale=1.0 / S)),
    ]


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML during a region."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.1):
        self.samples, self.power, self.reasons, self.max_mhz = [], [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # pragma: no cover - NVML absent
            self._nv = None
        self.period = period_s

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.power.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        out = {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}
        if self.power:
            out["power_w_median"] = round(statistics.median(self.power), 1)
            out["power_w_max"] = round(max(self.power), 1)
        return out


# --------------------------------------------------------------- GPU arm
def make_inputs(n_units: int, device, seed: int):
    """Seeded N(0,1) bf16 inputs for this rank's units, generated on device."""
    g = torch.Generator(device=device).manual_seed(seed)
    shp = (1, n_units, S, D)
    return [torch.randn(shp, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
            for _ in range(3)]


def traffic_from_profile(name: str, key: str = "traffic_bytes_per_launch_full"):
    """DRAM bytes per launch recorded in the committed ncu summary
    ``profiles/<name>.txt`` (line ``<key>: <bytes>``), if present."""
    p = os.path.join(ROOT, "profiles", f"{name}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def cpu_oracle_sample(target_s: float, max_units: int):
    """Time the oracle (reference algorithm, fp32, host cores) on a sample of units."""
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1234)
    vs = variants()
    flops_unit = 2 * 4 * D * S * S  # both operators, full mask
    # one unit first, to size the sample
    q, k, v = (torch.randn(1, 1, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    t0 = time.perf_counter()
    for name, _, kw in vs:
        oracle.run_op(name, q, k, v, **kw)
    one = time.perf_counter() - t0
    n = max(1, min(max_units, int(target_s / max(one, 1e-3))))
    q, k, v = (torch.randn(1, n, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    t0 = time.perf_counter()
    for name, _, kw in vs:
        oracle.run_op(name, q, k, v, **kw)
    dt = time.perf_counter() - t0
    return {"value": flops_unit * n / dt / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "sample_units": n, "seconds": round(dt, 3),
            "sample": f"{n} of {B_TOTAL * H_TOTAL} (batch, head) units of config 5, both operators, "
                      f"fp32 eager restatement on the host CPU"}


def cpu_config1():
    """BASELINE config 1 as the reference runs it: softcap (cap 50), non-causal,
    fp32, B1 H8 S512 D64, through the eager restatement on the host cores;
    median of 5 after one warm-up."""
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 8, 512, 64, generator=g) for _ in range(3))
    kw = dict(cap=50.0, causal=False)
    oracle.run_op("softcap_gemma2", q, k, v, **kw)
    ts = []
    for _ in range(5):
        t0 = time.perf_counter()
        oracle.run_op("softcap_gemma2", q, k, v, **kw)
        ts.append(time.perf_counter() - t0)
    ms = statistics.median(ts) * 1e3
    fl = 4 * 64 * 512 * 512 * 8
    return {"ms": round(ms, 3), "gflops": round(fl / ms / 1e6, 2),
            "cores": torch.get_num_threads(),
            "what": "softcap cap 50, non-causal, fp32, B1 H8 S512 D64, eager restatement"}


def _flat_param(values: torch.Tensor, lo: int, hi: int, H: int) -> torch.Tensor:
    """Per-head parameter of flattened (batch, head) units lo..hi-1 (unit u is head u % H)."""
    return values[torch.arange(lo, hi) % H]


def headline_suite(device, rank: int = 0, ws: int = 1, profile_launches: bool = False):
    """All ten operators at the north-star shape B4 H16 S4096 D128 (+ configs
    1-3 at N=1). The B*H units are split over the ranks like config 5 (each
    rank runs its contiguous range of (batch, head) units, per-head
    parameters follow their head); a variant's time is the maximum over ranks
    of its CUDA-event time. Inputs that fit in L2 rotate over enough copies
    that every launch reads from HBM.

    ``profile_launches``: launch each headline variant and config 2 exactly
    once, untimed, in the suite's order (for one ncu capture per variant)."""
    import chia_proj_b200 as cp
    pk, src = peaks()
    p_tensor = pk.get("bf16_tflops", FALLBACK["bf16_tflops"])
    hbm = pk.get("hbm_gbs", FALLBACK["hbm_gbs"])
    out = {}

    def make_sets(units, Sx, Dx, dtype, seed):
        by = 3 * units * Sx * Dx * 2
        n = 1 if by > L2_BYTES else min(8, math.ceil(4 * L2_BYTES / by))
        g = torch.Generator(device=device).manual_seed(seed)
        return [tuple(torch.randn(1, units, Sx, Dx, generator=g, device=device).to(dtype)
                      for _ in range(3)) for _ in range(n)]

    def bench_one(fn, sets, mask, units_total, Sx, Dx, iters=10, profile=None):
        if profile_launches:
            fn(*sets[0])
            torch.cuda.synchronize()
            return {"launched": 1}
        for i in range(3):
            fn(*sets[i % len(sets)])
        torch.cuda.synchronize()
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)

        def timed(n):
            device_lead(n)
            e0.record()
            for i in range(n):
                fn(*sets[i % len(sets)])
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1)

        # Short launches are timed again over enough launches that the timed
        # region lasts at least SUITE_MIN_MS (no collective depends on it).
        t_ms = timed(iters)
        if t_ms < SUITE_MIN_MS:
            iters = min(SUITE_MAX_ITERS, math.ceil(iters * SUITE_MIN_MS / max(t_ms, 1e-3)))
            t_ms = timed(iters)
        ms = max_over_ranks(t_ms / iters, device, ws)
        fl = 4 * Dx * cp.visible_pairs(mask, Sx) * units_total
        by = 4 * units_total * Sx * Dx * 2
        tf = fl / ms / 1e9
        ai = fl / by
        attainable = min(p_tensor, ai * hbm / 1e3)
        r = {"us": round(ms * 1e3, 1), "tflops": round(tf, 1),
             "pct_spec_peak": round(100 * tf / ws / SPEC_BF16_TFLOPS, 1),
             "hbm_gbs": round(by / ms / 1e6, 1),
             "bound": "hbm" if ai * hbm / 1e3 < p_tensor else "tensor",
             "frac": round(tf / ws / attainable, 3),
             "input_sets": len(sets), "timed_launches": iters}
        if profile is not None:
            dram = traffic_from_profile(profile, "traffic_bytes_per_launch")
            if dram is not None:
                r["dram_bytes"] = dram
                r["profile"] = f"profiles/{profile}.txt"
        return r

    B, H, Sx, Dx = 4, 16, 4096, 128
    U = B * H
    lo, hi = shard(U, ws, rank)
    sets = make_sets(hi - lo, Sx, Dx, torch.bfloat16, 7 + rank)
    gh = torch.Generator().manual_seed(0)
    tau = 0.5 + 1.5 * torch.rand(H, generator=gh)
    slopes = _flat_param(cp.alibi_slopes_geometric(H), lo, hi, H)
    temps = _flat_param(1.0 / tau, lo, hi, H)
    suite = {
        "softcap_gemma2": (lambda q, k, v: cp.softcap_gemma2(q, k, v, cap=50.0), cp.CAUSAL,
                           "cap 50, causal"),
        "bias_sliding_window": (cp.bias_sliding_window, cp.op_config("bias_sliding_window"),
                                "window 256"),
        "bias_local": (cp.bias_local, cp.op_config("bias_local"), "|i-j|<256"),
        "bias_alibi": (lambda q, k, v: cp.bias_alibi(q, k, v, slopes=slopes),
                       cp.CAUSAL, "slopes 2^(-8(h+1)/H), causal"),
        "bias_block_diagonal": (lambda q, k, v: cp.bias_block_diagonal(q, k, v, block=256),
                                cp.op_config("bias_block_diagonal", block=256), "block 256, causal"),
        "bias_dilated": (cp.bias_dilated, cp.op_config("bias_dilated"), "dilation 4, causal"),
        "bias_prefix_lm": (lambda q, k, v: cp.bias_prefix_lm(q, k, v, prefix=1024),
                           cp.op_config("bias_prefix_lm", prefix=1024), "prefix 1024"),
        "temp_perhead": (lambda q, k, v: cp.temp_perhead(q, k, v, temps=temps), cp.CAUSAL,
                         "1/tau_h, tau ~ U[0.5,2], causal"),
        "sigmoid_attn": (lambda q, k, v: cp.sigmoid_attn(q, k, v, causal=False,
                                                         bias=-math.log(Sx)), cp.FULL,
                         "bias -log S, non-causal"),
        "relu_attn": (lambda q, k, v: cp.relu_attn(q, k, v, causal=False, out_scale=1.0 / Sx),
                      cp.FULL, "1/S, non-causal"),
    }
    shape = {"B": B, "H": H, "S": Sx, "D": Dx, "dtype": "bf16", "units_per_gpu": hi - lo}
    with ClockSampler(torch.cuda.current_device()) as clk:
        res = {name: {**bench_one(fn, sets, m, U, Sx, Dx, profile=f"{name}_headline"),
                      "params": desc}
               for name, (fn, m, desc) in suite.items()}
    out["headline"] = {"shape": shape, "variants": res, "clocks": clk.summary(),
                       "peaks": f"{src}: bf16 burst {p_tensor} TFLOP/s, HBM {hbm} GB/s"}
    del sets
    if ws > 1:
        torch.cuda.empty_cache()
        return out
    if profile_launches:
        B2, H2, S2, D2 = 4, 16, 2048, 64
        sets = make_sets(B2 * H2, S2, D2, torch.bfloat16, 11)
        out["config2"] = bench_one(cp.bias_sliding_window, sets[:1],
                                   cp.op_config("bias_sliding_window"), B2 * H2, S2, D2)
        return out
    with ClockSampler(torch.cuda.current_device()) as clk:
        # config 2: causal window 256, D=64 (67 MB: rotated over 8 input sets)
        B2, H2, S2, D2 = 4, 16, 2048, 64
        sets = make_sets(B2 * H2, S2, D2, torch.bfloat16, 11)
        out["config2"] = {"shape": {"B": B2, "H": H2, "S": S2, "D": D2, "dtype": "bf16"},
                          "bias_sliding_window": bench_one(
                              cp.bias_sliding_window, sets, cp.op_config("bias_sliding_window"),
                              B2 * H2, S2, D2, iters=40, profile="bias_sliding_window_config2")}
        del sets
        # config 3: fp16 ALiBi / temperature, B8 H32 S4096 D128
        B3, H3 = 8, 32
        sets = make_sets(B3 * H3, 4096, 128, torch.float16, 13)
        tau3 = 0.5 + 1.5 * torch.rand(H3, generator=torch.Generator().manual_seed(0))
        sl3 = _flat_param(cp.alibi_slopes_geometric(H3), 0, B3 * H3, H3)
        te3 = _flat_param(1.0 / tau3, 0, B3 * H3, H3)
        out["config3"] = {"shape": {"B": B3, "H": H3, "S": 4096, "D": 128, "dtype": "fp16"},
                          "bias_alibi": bench_one(
                              lambda q, k, v: cp.bias_alibi(q, k, v, slopes=sl3),
                              sets, cp.CAUSAL, B3 * H3, 4096, 128, iters=5),
                          "temp_perhead": bench_one(
                              lambda q, k, v: cp.temp_perhead(q, k, v, temps=te3),
                              sets, cp.CAUSAL, B3 * H3, 4096, 128, iters=5)}
        del sets
        # config 1 on the GPU: fp32 inputs (converted to bf16 inside the call)
        g1 = torch.Generator(device=device).manual_seed(1)
        sets = [tuple(torch.randn(1, 8, 512, 64, generator=g1, device=device)
                      for _ in range(3)) for _ in range(8)]
        c1 = bench_one(lambda q, k, v: cp.softcap_gemma2(q, k, v, cap=50.0, causal=False),
                       sets, cp.FULL, 8, 512, 64, iters=50)
        c1["note"] = "fp32 inputs, computed in bf16 on the tensor cores; launch-latency bound"
        out["config1"] = {"shape": {"B": 1, "H": 8, "S": 512, "D": 64, "dtype": "fp32"},
                          "softcap_gemma2": c1}
        del sets
        out["decode"] = decode_bench(device)
        out["backward"] = backward_bench(device)
    out["configs_clocks"] = clk.summary()
    torch.cuda.empty_cache()
    return out


def decode_bench(device, iters: int = 100):
    """Decode step of a grouped-query model: one new query per sequence over
    8192 cached keys, B8, 32 query heads on 4 K/V heads, D128 bf16, causal
    (every cached key visible). HBM-bound: the bytes are K and V, read once.
    Timed on the split-KV decode kernel and, for comparison, on the tiled
    kernel (split_kv=False); three input sets rotate (134 MB each)."""
    import chia_proj_b200 as cp
    B, H, Hkv, Skv, D_ = 8, 32, 4, 8192, 128
    g = torch.Generator(device=device).manual_seed(5)
    sets = [(torch.randn(B, H, 1, D_, generator=g, device=device).to(torch.bfloat16),
             torch.randn(B, Hkv, Skv, D_, generator=g, device=device).to(torch.bfloat16),
             torch.randn(B, Hkv, Skv, D_, generator=g, device=device).to(torch.bfloat16))
            for _ in range(3)]
    mask = cp.Mask(left=-1, right=Skv - 1)
    pk, _ = peaks()
    hbm = pk.get("hbm_gbs", FALLBACK["hbm_gbs"])
    res = {"shape": {"B": B, "H": H, "H_kv": Hkv, "S_q": 1, "S_kv": Skv, "D": D_,
                     "dtype": "bf16"}}
    by = 2 * B * Hkv * Skv * D_ * 2 + 2 * B * H * D_ * 2
    fl = 4 * D_ * Skv * B * H
    for name, split in (("split_kv", True), ("tiled", False)):
        fn = lambda q, k, v: cp.attention(q, k, v, mask=mask, split_kv=split)
        for i in range(3):
            fn(*sets[i % 3])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        device_lead(iters)
        e0.record()
        for i in range(iters):
            fn(*sets[i % 3])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        res[name] = {"us": round(ms * 1e3, 1), "hbm_gbs": round(by / ms / 1e6, 1),
                     "frac_hbm": round(by / ms / 1e6 / hbm, 3),
                     "tflops": round(fl / ms / 1e9, 2)}
    del sets
    return res


def backward_bench(device, iters: int = 10):
    """Backward pass (dQ, dK, dV) at the headline shape B4 H16 S4096 D128
    bf16: the kernel call chia_attn_bwd given the forward's output and
    log-sum-exp. Mask-aware FLOPs of the backward: five products (S, dP, dV,
    dK, dQ) of 2 * D per visible pair, 10 * D * pairs * B * H."""
    import chia_proj_b200 as cp
    B, H, Sx, Dx = 4, 16, 4096, 128
    g = torch.Generator(device=device).manual_seed(17)
    q, k, v, do = (torch.randn(B, H, Sx, Dx, generator=g, device=device).to(torch.bfloat16)
                   for _ in range(4))
    pk, _ = peaks()
    p_tensor = pk.get("bf16_tflops", FALLBACK["bf16_tflops"])
    res = {"shape": {"B": B, "H": H, "S": Sx, "D": Dx, "dtype": "bf16"}}
    cases = {
        "softcap_gemma2": (dict(mod="softcap", softcap=50.0, mask=cp.CAUSAL), cp.CAUSAL),
        "bias_prefix_lm": (dict(mask=cp.op_config("bias_prefix_lm", prefix=1024)),
                           cp.op_config("bias_prefix_lm", prefix=1024)),
        "sigmoid_attn": (dict(norm="sigmoid", sig_bias=-math.log(Sx), mask=cp.FULL), cp.FULL),
    }
    for name, (kw, mask) in cases.items():
        if kw.get("norm", "softmax") == "softmax":
            o, lse = cp.attention(q, k, v, return_lse=True, **kw)
        else:
            o, lse = cp.attention(q, k, v, **kw), None
        fn = lambda: cp.attention_backward(do, q, k, v, o, lse, **kw)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        fl = 10 * Dx * cp.visible_pairs(mask, Sx) * B * H
        res[name] = {"us": round(ms * 1e3, 1), "tflops": round(fl / ms / 1e9, 1),
                     "frac": round(fl / ms / 1e9 / p_tensor, 3)}
    del q, k, v, do
    return res


def profile_bwd_decode(device):
    """One backward call (B4 H16 S4096 D128 bf16, softcap 50, causal) and one
    decode call (the decode benchmark's shape), each after one untimed call."""
    import chia_proj_b200 as cp
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(17)
    q, k, v, do = (torch.randn(4, 16, 4096, 128, generator=g, device=device).to(torch.bfloat16)
                   for _ in range(4))
    kw = dict(mod="softcap", softcap=50.0, mask=cp.CAUSAL)
    o, lse = cp.attention(q, k, v, return_lse=True, **kw)
    for _ in range(2):
        cp.attention_backward(do, q, k, v, o, lse, **kw)
    del q, k, v, do, o, lse
    qd = torch.randn(8, 32, 1, 128, generator=g, device=device).to(torch.bfloat16)
    kd, vd = (torch.randn(8, 4, 8192, 128, generator=g, device=device).to(torch.bfloat16)
              for _ in range(2))
    for _ in range(2):
        cp.attention(qd, kd, vd, mask=cp.Mask(left=-1, right=8191))
    torch.cuda.synchronize()
    print(json.dumps({"profiled": ["fmha_bwd_kernel", "decode_kernel"]}))


def preheat(step, seconds: float):
    """Untimed load before the warm-up steps, so that every N reaches the
    power state of a long run (at the 1 kW cap the SM clock settles lower
    than in a short burst) before its timed region."""
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds:
        step()
        torch.cuda.synchronize()
        n += 1
    return n


def e2e_overlapped(vs, host_in, host_out, device, chunk_units: int, steps: int, ws: int,
                   barrier):
    """Same two operators through the public API from pinned host buffers:
    each step copies every chunk of units host->device, runs both operators
    on it and copies both outputs back, on three streams so that the copies
    of chunk c+1 (in) and c-1 (out) overlap the compute of chunk c. Returns
    the device time of ``steps`` steps (max over ranks), in ms."""
    n = host_in[0].shape[1]
    chunks = [(a, min(n, a + chunk_units)) for a in range(0, n, chunk_units)]
    cu = min(chunk_units, n)
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    dev_in = [[torch.empty((1, cu, S, D), dtype=torch.bfloat16, device=device)
               for _ in range(3)] for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    main = torch.cuda.current_stream(device)

    def step():
        for ci, (a, b) in enumerate(chunks):
            slot = ci % 2
            s_in.wait_event(ev_done[slot])  # the chunk two back is done with this slot
            with torch.cuda.stream(s_in):
                xs = [t[:, :b - a] for t in dev_in[slot]]
                for t, h in zip(xs, host_in):
                    t.copy_(h[:, a:b], non_blocking=True)
                ev_in[slot].record(s_in)
            s_cmp.wait_event(ev_in[slot])
            s_cmp.wait_event(ev_out[slot])  # outputs of the chunk two back are copied out
            with torch.cuda.stream(s_cmp):
                outs = [(name, fn(*xs)) for name, fn, _ in vs]
                ev_done[slot].record(s_cmp)
            s_out.wait_event(ev_done[slot])
            with torch.cuda.stream(s_out):
                for name, o in outs:
                    host_out[name][:, a:b].copy_(o, non_blocking=True)
                    o.record_stream(s_out)
                ev_out[slot].record(s_out)

    def run(k):
        for st in (s_in, s_cmp, s_out):
            st.wait_stream(main)
        for _ in range(k):
            step()
        for st in (s_in, s_cmp, s_out):
            main.wait_stream(st)

    run(1)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record(main)
    run(steps)
    e1.record(main)
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(e0.elapsed_time(e1), device, ws)


def run_ours(a):
    import torch.distributed as dist

    import chia_proj_b200 as cp

    ws, rank, local = dist_env()
    assert ws == a.gpus, f"--gpus {a.gpus} but WORLD_SIZE {ws}"
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import datetime
        # stdout carries exactly one JSON line: NCCL's own log goes to stderr
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    units = a.units
    lo, hi = shard(units, ws, rank)
    n = hi - lo
    q, k, v = make_inputs(n, device, seed=1000 + rank)
    outs = {}
    vs = variants()
    fl_unit = 4 * D * cp.visible_pairs(cp.FULL, S)
    flops_step_total = fl_unit * units * len(vs)
    stream = torch.cuda.current_stream(device)

    def step(events=None):
        for vi, (name, fn, _) in enumerate(vs):
            if events is not None:
                events[vi][0].record(stream)
            outs[name] = fn(q, k, v)
            if events is not None:
                events[vi][1].record(stream)

    def barrier():
        if ws > 1:
            dist.barrier()

    preheat_steps = preheat(step, a.preheat_seconds) if a.preheat_seconds > 0 else 0
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    cp.check_device_status(local)

    ev = [[[torch.cuda.Event(True), torch.cuda.Event(True)] for _ in vs] for _ in range(a.steps)]
    e_start, e_end = torch.cuda.Event(True), torch.cuda.Event(True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e_start.record(stream)
        for s in range(a.steps):
            step(ev[s])
        e_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = e_start.elapsed_time(e_end)
    per_kernel_ms = {name: statistics.mean(ev[s][vi][0].elapsed_time(ev[s][vi][1])
                                           for s in range(a.steps))
                     for vi, (name, _, _) in enumerate(vs)}
    cp.check_device_status(local)

    ms_max = max_over_ranks(ms, device, ws)
    value = flops_step_total * a.steps / (ms_max * 1e-3) / 1e12
    csum = clk.summary()
    # per-rank clock / power record, gathered to rank 0 (after timing)
    rank_clk = gather_all([csum.get("sm_mhz") or 0.0, csum.get("power_w_median", 0.0),
                           csum.get("power_w_max", 0.0)], device, ws)

    # ---- verification: one unit per rank against an fp32 torch reference,
    # errors gathered to rank 0 after timing
    with torch.no_grad():
        errs = []
        for name, _, kw in vs:
            qf, kf, vf = (x[0, 0].float() for x in (q, k, v))
            s_ = (qf @ kf.t()) / math.sqrt(D)
            p_ = torch.sigmoid(s_ + kw["bias"]) if name == "sigmoid_attn" else \
                torch.relu(s_) * kw["out_scale"]
            ref = p_ @ vf
            errs.append((outs[name][0, 0].float() - ref).abs().max().item())
            del s_, p_, ref
    e = gather_max(errs, device, ws)
    verify = {name: e[i] for i, (name, _, _) in enumerate(vs)}

    # ---- end to end through the public API, host buffers, every step
    e2e = None
    if not a.no_e2e:
        host_in = [x.cpu().pin_memory() for x in (q, k, v)]
        host_out = {name: torch.empty(q.shape, dtype=q.dtype).pin_memory() for name, _, _ in vs}
        del q, k, v
        outs.clear()
        torch.cuda.empty_cache()
        e2e_steps = max(1, a.e2e_steps)
        e2e_ms = e2e_overlapped(vs, host_in, host_out, device, a.e2e_chunk, e2e_steps, ws,
                                barrier)
        bi = 3 * host_in[0].numel() * host_in[0].element_size()
        bo = len(vs) * host_in[0].numel() * host_in[0].element_size()
        e2e = {"value": round(flops_step_total * e2e_steps / (e2e_ms * 1e-3) / 1e12, 2),
               "unit": "TFLOP/s", "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
               "steps": e2e_steps,
               "path": f"chia_proj_b200.sigmoid_attn / relu_attn on chunks of {a.e2e_chunk} "
                       f"units: pinned host inputs copied in and both outputs copied out every "
                       f"step, copies of neighbouring chunks overlapping the compute"}

    suite = None
    if not a.no_suite:
        suite = headline_suite(device, rank, ws)

    result = None
    if rank == 0:
        pk, src = peaks()
        dom = max(per_kernel_ms, key=per_kernel_ms.get)
        achieved = fl_unit * n / (per_kernel_ms[dom] * 1e-3) / 1e12
        peak = pk.get("bf16_tflops_sustained", FALLBACK["bf16_tflops_sustained"])
        traffic = traffic_from_profile(f"{dom}_config5")
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": ws,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded N(0,1) q, k, v (no dataset in the reference)",
            "config": dict(CONFIG),
            "sharding": {"units_total": units, "units_per_gpu": n, "parallelism": f"bxh-shard{ws}",
                         "l2": "inputs 6.4 GB/N per GPU > 126 MB L2, no flush needed",
                         "preheat_steps": preheat_steps,
                         "preheat_seconds": a.preheat_seconds},
            "variants": {name: {"ms_per_launch": round(per_kernel_ms[name], 3),
                                "tflops_per_gpu": round(fl_unit * n / per_kernel_ms[name] / 1e9, 1),
                                "pct_spec_bf16_peak": round(100 * fl_unit * n / per_kernel_ms[name]
                                                            / 1e9 / SPEC_BF16_TFLOPS, 1),
                                "verify_max_abs": verify[name]}
                         for name, _, _ in vs},
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a "
                                        f"seconds-long region)",
                         "frac_of_spec_2250": round(achieved / SPEC_BF16_TFLOPS, 4),
                         "traffic": traffic},
            "clocks": csum,
            "clocks_per_rank": [{"rank": r, "sm_mhz": rank_clk[r][0],
                                 "power_w_median": rank_clk[r][1], "power_w_max": rank_clk[r][2]}
                                for r in range(ws)],
            "gpu_launches": len(vs) * a.steps,
            "e2e": e2e,
        }
        if suite is not None:
            result["suite"] = suite
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if ws == 1 and not a.no_cpu_baseline:
            cpu = cpu_oracle_sample(target_s=a.cpu_seconds, max_units=16)
            result["cpu_baseline"] = {**cpu, "kind": "port", "config1": cpu_config1()}
        print(json.dumps(result), flush=True)


def gather_all(vals, device, ws: int):
    """``vals`` of every rank, as a list indexed by rank."""
    e = torch.tensor(list(vals), dtype=torch.float64, device=device)
    if ws == 1:
        return [[float(x) for x in e]]
    import torch.distributed as dist
    gathered = [torch.zeros_like(e) for _ in range(ws)]
    dist.all_gather(gathered, e)
    return [[float(x) for x in g] for g in gathered]


# ------------------------------------------------------------ reference arm
def run_reference(a):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    vs = variants()
    g = torch.Generator().manual_seed(99)
    q, k, v = (torch.randn(1, 1, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    fl_unit = 2 * 4 * D * S * S

    def one_step(n):
        t0 = time.perf_counter()
        for i in range(n):
            for name, _, kw in vs:
                oracle.run_op(name, q, k, v, **kw)
        return time.perf_counter() - t0

    t1 = one_step(1)
    n = max(1, min(16, int(a.ref_step_seconds / max(t1, 1e-3))))
    for _ in range(max(0, a.warmup - 1)):
        one_step(n)
    times = [one_step(n) for _ in range(a.steps)]
    dt = sum(times) / len(times)
    value = fl_unit * n / dt / 1e12
    sample = (f"{n} (batch, head) unit(s) of config 5 per step (both operators, S=8192, D=128), "
              f"fp32 eager restatement of the reference on the host CPU")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1)",
        "config": dict(CONFIG),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-suite", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-step-seconds", type=float, default=3.0)
    ap.add_argument("--preheat-seconds", type=float, default=2.0,
                    help="untimed load before the warm-up steps (power state of a long run)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunk", type=int, default=64,
                    help="(batch, head) units per host<->device chunk in the e2e measurement")
    ap.add_argument("--suite-only", action="store_true",
                    help="run only the per-variant suite at the north-star shape (1 GPU)")
    ap.add_argument("--profile-launches", action="store_true",
                    help="launch each headline variant and config 2 once, untimed (ncu)")
    ap.add_argument("--profile-bwd-decode", action="store_true",
                    help="one backward call at the headline shape (softcap, causal) and one "
                         "decode call of the decode benchmark, untimed (ncu)")
    ap.add_argument("--units", type=int, default=B_TOTAL * H_TOTAL,
                    help="(batch, head) units in the job; smaller values are for ncu captures")
    a = ap.parse_args(argv)
    if a.warmup < 3 and a.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if a.impl == "reference":
        run_reference(a)
    elif a.profile_bwd_decode:
        profile_bwd_decode(torch.device("cuda", 0))
    elif a.suite_only or a.profile_launches:
        torch.cuda.set_device(0)
        print(json.dumps({"suite": headline_suite(torch.device("cuda", 0),
                                                  profile_launches=a.profile_launches)}),
              flush=True)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
