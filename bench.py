#!/usr/bin/env python3
"""Benchmark: post-prefill KV-cache compression on B200, sharded across the GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 4]

Workload (default): BASELINE config 4 -- Llama-3-70B-shaped 128K cache, 80 layers
x 8 KV heads x head_dim 128, batch 1, T=131072, fp16 (42.95 GB of K+V), RoPE base
5e5, 'max' preset: K2V2 + 80 % eviction with the key-key scorer on layer 0,
first/last 2 layers protected at fp16.  Synthetic data (seeded N(0,1) keys with
outlier channels + RoPE, N(0,1) values), generated on the device.  ``--config 2``
runs the real-attention scorer over every layer's 64 synthetic queries instead.

One step = score (each rank scores its block of KV heads; per-head column sums are
all-gathered over NCCL, or for the real scorer the per-rank sums are all-reduced) ->
keep set -> compress every layer (or head slice) the rank owns (one launch per half) +
fp16 gather of its share of the protected layers -> all-gather of the per-layer
compressed sizes.  Ranks own whole layers (sharding.make_plan, mode "auto"; head slices only
when every rank would keep 8 or more KV heads).  Strong scaling: the cache is fixed, N GPUs
share it.  value = fp16-in bytes of the
whole cache / max-over-ranks step time.  Inputs are far larger than L2, so no flush is
needed between steps.

The same JSON line carries the kernel-only compress and dequantize rooflines of this
configuration and (on one GPU) of configs 1-3, the end-to-end number through
``NexusQuantEvict(layout="compressed")`` on a cache in pinned host memory, the CPU
baseline, the entropy-coded size (zstd and rANS host post-steps, outside the timed region),
and (`extras`, one GPU) the device times of the tensor-core decode attention and merge
survivor search on the step's own data.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from nexusquant_b200 import entropy as E  # noqa: E402
from nexusquant_b200 import kernels as K  # noqa: E402
from nexusquant_b200 import sharding as S  # noqa: E402
from nexusquant_b200 import synthetic as syn  # noqa: E402
from nexusquant_b200.pipeline import NexusQuantEvict, kept_capacity, n_keep_for  # noqa: E402

METRIC = "KV compress GB/s (fp16 in) & dequant GB/s, % of HBM peak, at 1/2/4/8 B200"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def config_dict(cfg, cap: int, world: int) -> dict:
    """The workload description, identical in both arms' lines."""
    return {"workload": cfg.name, "layers": cfg.n_layers, "batch": cfg.batch, "heads": cfg.heads,
            "seq": cfg.seq, "head_dim": cfg.head_dim, "key_bits": cfg.key_bits, "value_bits": cfg.value_bits,
            "eviction_rate": cfg.eviction_rate, "scorer": cfg.scorer if cfg.eviction_rate > 0 else "none",
            "kept_tokens": cap, "protected_layers": sorted(S.protected_layers(cfg.n_layers, cfg.protect_boundary)),
            "parallelism": (f"head-sharded x{world}" if S.plan_mode(cfg.heads, world) == "heads"
                            else f"layer-sharded x{world}"),
            "l2": f"inputs ({cfg.fp16_bytes / 1e9:.2f} GB) larger than L2; no flush"}


def cap_for(cfg) -> int:
    if cfg.eviction_rate <= 0:
        return cfg.seq
    return kept_capacity(cfg.seq, cfg.sliding_window, n_keep_for(cfg.seq, cfg.sliding_window, cfg.eviction_rate))


# ------------------------------------------------------------------ clocks (NVML)
class ClockSampler:
    """Samples SM clock and clock-event reasons every ~5 ms on a background thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int):
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self.samples, self.reasons = [], 0
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(0.005)

    def sample(self):
        if not self.ok:
            return
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            pass

    def __enter__(self):
        self.sample()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.t.join()
        self.sample()

    def report(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2], "sm_max_mhz": self.max_mhz, "samples": len(s),
                "reasons": [n for b, n in self.REASONS.items() if self.reasons & b]}


class GpuLocalCpus:
    """Context: run on the CPUs NVML reports as local to the GPU, so pinned host buffers allocated
    and first touched inside land on the GPU's NUMA node (the e2e leg reads the cache across
    PCIe from them).  A no-op where NVML or the affinity call is unavailable."""

    def __init__(self, index: int):
        self.index, self.saved = index, None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            n = (os.cpu_count() + 63) // 64
            words = pynvml.nvmlDeviceGetCpuAffinity(h, n)
            cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
            cpus &= os.sched_getaffinity(0)
            if cpus:
                self.saved = os.sched_getaffinity(0)
                os.sched_setaffinity(0, cpus)
        except Exception:
            self.saved = None
        return self

    def __exit__(self, *a):
        if self.saved:
            os.sched_setaffinity(0, self.saved)


def timed(fn, steps, warmup, world, group=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=group)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms = float(t.item())
        dist.barrier(group=group)
    return ms


# -------------------------------------------------------------------------- shard
class Shard:
    """One rank's part of the compression of a benchmark cache."""

    def __init__(self, cfg, rank: int, world: int, device, group=None):
        self.cfg, self.rank, self.world, self.dev, self.group = cfg, rank, world, device, group
        L, h = cfg.n_layers, cfg.heads
        self.plan = S.make_plan(L, h, cfg.protect_boundary, rank, world)
        self.owned = list(self.plan.layers)
        self.quant = list(self.plan.quantized)
        self.prot = list(self.plan.protected)
        self.protected = S.protected_layers(L, cfg.protect_boundary)
        self.lh0, self.lh1 = self.plan.layer_heads      # heads of each owned layer
        self.hl = self.lh1 - self.lh0
        self.h0, self.h1, self.per = self.plan.head_begin, self.plan.head_end, self.plan.heads_per_rank
        self.real = cfg.scorer == "real" and cfg.eviction_rate > 0
        self.nk = n_keep_for(cfg.seq, cfg.sliding_window, cfg.eviction_rate)
        self.cap = cap_for(cfg)
        b, T, d = cfg.batch, cfg.seq, cfg.head_dim
        # resident data: this rank's layers (its head slice of them under the head plan)
        self.K, self.V, self.Q = {}, {}, {}
        for l in self.owned:
            k, v = syn.device_layer(cfg, l, device)
            self.K[l], self.V[l] = self._slice(k), self._slice(v)
            del k, v
            if self.real:
                self.Q[l] = self._slice(syn.device_queries(cfg, l, device))
        if self.real or cfg.eviction_rate <= 0:
            self.K0 = None
        elif self.plan.mode == "heads":
            self.K0 = self.K[0]  # the scored block is this rank's slice of layer 0
        else:
            k0 = self.K[0] if 0 in self.K else syn.device_layer(cfg, 0, device)[0]
            self.K0 = k0[:, self.h0:self.h1].contiguous() if self.h1 > self.h0 else None
        dp = K.next_pow2(d)
        self.levels = (2 ** cfg.key_bits, 2 ** cfg.value_bits)
        n = self.cap
        self.codes = [K.LayerCodes(
            torch.empty((b, self.hl, n, K.packed_bytes(dp, self.levels[0])), dtype=torch.uint8, device=device),
            torch.empty((b, self.hl, n, K.packed_bytes(dp, self.levels[1])), dtype=torch.uint8, device=device),
            torch.empty((b, self.hl, n), dtype=torch.float16, device=device),
            torch.empty((b, self.hl, n), dtype=torch.float16, device=device), *self.levels) for _ in self.quant]
        self.prot_out = {l: (torch.empty((b, self.hl, n, d), dtype=torch.float16, device=device),
                             torch.empty((b, self.hl, n, d), dtype=torch.float16, device=device)) for l in self.prot}
        self.gathered = torch.empty((world * b * self.per, T), dtype=torch.float32, device=device)
        pkv = K.packed_bytes(dp, self.levels[0]) + K.packed_bytes(dp, self.levels[1]) + 4
        self.sizes = S.local_layer_sizes(self.plan, [b * self.hl * n * pkv] * len(self.quant),
                                         [2 * b * self.hl * n * d * 2] * len(self.prot), device=device)
        self.sizes_all = torch.zeros((world * L,), dtype=torch.int64, device=device)
        self.kept_idx = torch.arange(n, dtype=torch.int32, device=device).expand(b, n).contiguous()
        self.kept_count = torch.full((b,), n, dtype=torch.int32, device=device)
        self.launches = 0

    def _slice(self, t: torch.Tensor) -> torch.Tensor:
        return t if self.hl == t.shape[1] else t[:, self.lh0:self.lh1].contiguous()

    def compress_algo_bytes(self) -> int:
        """Algorithmic bytes of this rank's compress launch: read 2*d bytes per kept K and V
        row, write packed codes + fp16 scale per row, read the kept index per (row, head) once."""
        b, d = self.cfg.batch, self.cfg.head_dim
        dp = K.next_pow2(d)
        pk, pv = K.packed_bytes(dp, self.levels[0]), K.packed_bytes(dp, self.levels[1])
        return len(self.quant) * b * self.hl * self.cap * (2 * d * 2 + pk + pv + 4)

    def importance(self, k_scored=None):
        """Importance [b, T] on every rank: key-key over the scored block of layer 0 (per-head
        column sums all-gathered), or the real scorer over this rank's layers/heads (sums
        all-reduced).  k_scored: the block of layer-0 keys to score (default the resident one)."""
        cfg = self.cfg
        b, h, T = cfg.batch, cfg.heads, cfg.seq
        if self.real:
            acc = torch.zeros((b, T), dtype=torch.float32, device=self.dev)
            for l in self.owned:
                K.score_attention(self.Q[l], self.K[l], T - self.Q[l].shape[2], out=acc, accumulate=True)
                self.launches += 3
            # score_attention averages over the call's query heads: weight this rank's share
            acc *= self.Q[self.owned[0]].shape[1] / (cfg.q_heads or h) if self.owned else 0.0
            if self.world > 1:
                dist.all_reduce(acc, group=self.group)
            return acc / cfg.n_layers
        k0 = self.K0 if k_scored is None else k_scored
        if self.h1 > self.h0:
            ph = K.score_keykey(k0, 32, per_head=True)
            self.launches += 3
        else:
            ph = torch.zeros((b, 0, T), dtype=torch.float32, device=self.dev)
        allh = S.gather_head_scores(ph, self.plan, self.group, self.gathered)
        self.launches += 1
        return K.reduce_heads(allh, float(h))

    def step(self):
        cfg = self.cfg
        # global index of the compressed cache: the per-layer byte sizes of fixed-capacity
        # outputs are known up front, so their exchange overlaps scoring and compression
        _, sizes_work = S.gather_layer_index(self.sizes, self.plan, self.group, self.sizes_all, async_op=True)
        if cfg.eviction_rate > 0:
            imp = self.importance()
            idx, cnt = K.select_keep(imp, cfg.sliding_window, self.nk)
            self.launches += 1
            self.kept_idx, self.kept_count = idx[:, :self.cap], cnt
        if self.quant:
            K.compress_layers([self.K[l] for l in self.quant], [self.V[l] for l in self.quant],
                              key_levels=self.levels[0], value_levels=self.levels[1], kept_idx=self.kept_idx,
                              kept_count=self.kept_count, n_kept=self.cap, rope_base=cfg.rope_base,
                              rope_rows=cfg.seq, codes_out=self.codes)
            self.launches += 2 * math.ceil(len(self.quant) / 96)  # key and value kernels
        for l in self.prot:
            K.gather_rows(self.K[l], self.kept_idx, self.cap, self.kept_count, out=self.prot_out[l][0])
            K.gather_rows(self.V[l], self.kept_idx, self.cap, self.kept_count, out=self.prot_out[l][1])
            self.launches += 2
        if sizes_work is not None:
            sizes_work.wait()

    def compress_only(self):
        K.compress_layers([self.K[l] for l in self.quant], [self.V[l] for l in self.quant],
                          key_levels=self.levels[0], value_levels=self.levels[1], kept_idx=self.kept_idx,
                          kept_count=self.kept_count, n_kept=self.cap, rope_base=self.cfg.rope_base,
                          rope_rows=self.cfg.seq, codes_out=self.codes)

    def dequant(self, outs):
        return K.decompress_layers(self.codes, self.kept_idx, head_dim=self.cfg.head_dim, count=self.kept_count,
                                   rope_base=self.cfg.rope_base, rope_rows=self.cfg.seq, out_k=outs[0],
                                   out_v=outs[1])

    def free(self):
        self.K.clear()
        self.V.clear()
        self.Q.clear()
        self.K0 = None


def kernel_rooflines(sh: Shard, steps: int, peak: float) -> dict:
    """Kernel-only compress and dequantize of the shard's quantized layers (CUDA events on the
    launching stream, inputs far larger than L2)."""
    if not sh.quant:
        return {}
    kms = timed(sh.compress_only, steps, 2, 1) / steps
    cfg = sh.cfg
    outs = ([torch.empty((cfg.batch, sh.hl, sh.cap, cfg.head_dim), dtype=torch.float16, device=sh.dev)
             for _ in sh.quant],
            [torch.empty((cfg.batch, sh.hl, sh.cap, cfg.head_dim), dtype=torch.float16, device=sh.dev)
             for _ in sh.quant])
    dms = timed(lambda: sh.dequant(outs), steps, 2, 1) / steps
    del outs
    algo = sh.compress_algo_bytes()
    c = algo / (kms / 1e3) / 1e9
    dq = algo / (dms / 1e3) / 1e9
    return {"compress": {"achieved": round(c, 1), "frac": round(c / peak, 4), "launch_ms": round(kms, 4),
                         "algo_bytes": algo},
            "dequant": {"achieved": round(dq, 1), "frac": round(dq / peak, 4), "launch_ms": round(dms, 4),
                        "algo_bytes": algo}}


def per_config_rooflines(skip: int, dev, steps: int, peak: float) -> dict:
    """Kernel-only compress / dequantize rooflines of configs 1-3 at their own shapes on this GPU
    (one full cache each, keep set from the configuration's scorer)."""
    out = {}
    for cid in (1, 2, 3):
        if cid == skip:
            continue
        cfg = syn.CONFIGS[cid]
        sh = Shard(cfg, 0, 1, dev)
        sh.step()
        torch.cuda.synchronize()
        r = kernel_rooflines(sh, max(5, min(steps, 20)), peak)
        r["config"] = {"workload": cfg.name, "layers": cfg.n_layers, "batch": cfg.batch, "heads": cfg.heads,
                       "seq": cfg.seq, "head_dim": cfg.head_dim, "kept_tokens": sh.cap}
        out[f"config{cid}"] = r
        sh.free()
        del sh
        torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------- CPU leg
def cpu_sample(cfg, seconds_hint: float = 15.0):
    """Time the oracle port on this host: score layer 0 (all heads, float64) + select +
    compress of 2 quantized layers' kept rows; extrapolate to the whole cache.  Returns
    (GB/s fp16-in, threads, description)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    orc.lib()
    b, h, T, d = cfg.batch, cfg.heads, cfg.seq, cfg.head_dim
    g = torch.Generator().manual_seed(7)
    k0 = torch.randn(b, h, T, d, generator=g)
    t0 = time.perf_counter()
    obs = 32
    scale = float(np.float32(d ** -0.5))
    k0n = k0.numpy()

    def one(hi):
        return orc.attn_colsum(k0n[0, hi, T - obs:], k0n[0, hi], scale)
    with ThreadPoolExecutor(threads) as ex:
        cols = list(ex.map(one, range(h)))
    imp = (np.sum(cols, 0) / h)[None]
    m = orc.keep_mask(imp, T, cfg.sliding_window, cfg.eviction_rate)
    t_score = time.perf_counter() - t0
    kept = np.nonzero(m[0])[0]
    n = len(kept)
    cos, sin = orc.rope_tables(kept, d, cfg.rope_base)
    cr, sr = np.tile(cos, (h, 1)), np.tile(sin, (h, 1))
    rows = torch.randn(2, h * n, d, generator=g).numpy()
    t1 = time.perf_counter()
    for _ in range(2):
        kc, ks = orc.quantize(rows[0], K.next_pow2(d), 2 ** cfg.key_bits, cr, sr)
        vc, vs = orc.quantize(rows[1], K.next_pow2(d), 2 ** cfg.value_bits)
        orc.pack(kc, 2 ** cfg.key_bits)
        orc.pack(vc, 2 ** cfg.value_bits)
    t_layer = (time.perf_counter() - t1) / 2
    n_q = cfg.n_layers - 2 * cfg.protect_boundary
    total = t_score + n_q * t_layer
    gbs = cfg.fp16_bytes / total / 1e9
    desc = (f"oracle port (C, OpenMP {threads} threads): key-key score of layer 0 ({h} heads x {T} tokens, "
            f"float64) + keep set, measured {t_score:.2f}s; compress of 2 quantized layers' kept rows "
            f"({n} tokens x {h} heads, K+V) measured {t_layer:.3f}s/layer; extrapolated to {n_q} quantized "
            f"layers (protected-layer copies not counted)")
    return gbs, threads, desc


# ------------------------------------------------------------------------ e2e
class _Cache:
    def __init__(self, ks, vs):
        self.key_cache, self.value_cache = list(ks), list(vs)


def e2e_leg(sh: Shard, steps: int):
    """End to end through the drop-in API: NexusQuantEvict(layout="compressed", device=...,
    result_on_host=True).compress(cache) on this rank's share of the cache held in pinned host
    memory.  Per step: the scored keys cross PCIe to the device (on one GPU the API copies
    layer 0's keys itself; with several ranks each copies its scored block and the importance,
    sharded as in the device step, is handed to compress()), only the kept rows of every layer
    cross PCIe (gather kernel), and the compressed cache comes back to pinned host memory group
    by group while the next group is processed."""
    cfg = sh.cfg
    dev = sh.dev
    if sh.real:
        return None, "the real scorer needs the model's queries; e2e is measured on the key-key configs"
    try:
        host = {l: (torch.empty(sh.K[l].shape, dtype=sh.K[l].dtype, pin_memory=True),
                    torch.empty(sh.V[l].shape, dtype=sh.V[l].dtype, pin_memory=True)) for l in sh.owned}
    except RuntimeError as e:
        return None, f"pinned host allocation failed: {e}"
    for l in sh.owned:
        host[l][0].copy_(sh.K[l])
        host[l][1].copy_(sh.V[l])
    torch.cuda.synchronize()
    single = sh.world == 1
    k0_host = None
    if not single and sh.K0 is not None:
        k0_host = torch.empty(sh.K0.shape, dtype=sh.K0.dtype, pin_memory=True)
        k0_host.copy_(sh.K0)
    # the device copies of the rank's layers are not used by this leg: free them
    sh.free()
    torch.cuda.empty_cache()
    cache = _Cache([host[l][0] for l in sh.owned], [host[l][1] for l in sh.owned])
    prot_local = {i for i, l in enumerate(sh.owned) if l in sh.protected}
    ev = NexusQuantEvict(bits=cfg.key_bits, key_bits=cfg.key_bits, value_bits=cfg.value_bits,
                         eviction_rate=cfg.eviction_rate, sliding_window=cfg.sliding_window, obs_window=32,
                         rope_base=cfg.rope_base, protect_boundary=0, protected_layers=prot_local,
                         layout="compressed", device=dev, result_on_host=True, group_layers=8)
    k0_dev = None if k0_host is None else torch.empty(k0_host.shape, dtype=k0_host.dtype, device=dev)
    b, T, d = cfg.batch, cfg.seq, cfg.head_dim
    row = d * 2  # fp16 row bytes
    scored = b * (sh.h1 - sh.h0) * T * row if (single or k0_host is not None) else 0
    h2d = scored + len(sh.owned) * 2 * b * sh.hl * sh.cap * row
    out = {}

    def step():
        if single:
            res, _ = ev.compress(cache)
        else:
            if k0_dev is not None:
                k0_dev.copy_(k0_host, non_blocking=True)
            imp = sh.importance(k0_dev)
            res, _ = ev.compress(cache, importance=imp)
        out["res"] = res

    step()
    torch.cuda.synchronize()
    res = out["res"]
    d2h = res.nbytes() + res.kept_count.numel() * 4
    each = [round(timed(step, 1, 0, sh.world, sh.group), 1) for _ in range(2)]  # warm-up, per step
    ms = timed(step, steps, 0, sh.world, sh.group)
    e2e = {"value": round(cfg.fp16_bytes * steps / (ms / 1e3) / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
           "ms_per_step": round(ms / steps, 3), "warmup_ms": each,
           "path": "NexusQuantEvict(layout='compressed', device=cuda, result_on_host=True).compress(cache) on a "
                   "cache in pinned host memory; kept rows gathered over PCIe, codes copied back per 8 layers"}
    return (e2e, res), None


def entropy_leg(cache, cfg, max_tokens: int = 2048) -> dict:
    """zstd (level 22, system libzstd) of the temporal-delta streams of one quantized layer's first
    ``max_tokens`` kept tokens: the reference's reported host post-step, outside every timed region."""
    q = [i for i, l in enumerate(cache.layers) if not l.protected]
    if not q:
        return {"error": "no quantized layer"}
    r = E.entropy_report(cache, level=22, layers=[q[0]], max_tokens=max_tokens, threads=os.cpu_count() or 1)
    n_sym_total = sum(2 * cache.batch * l.codes.k_codes.shape[1] * cache.n_kept * cache.head_dim_padded
                      for l in cache.layers if not l.protected)
    idx_bytes = r["bits_per_symbol"] / 8.0 * n_sym_total
    other = sum(l.nbytes() - (l.codes.k_codes.numel() + l.codes.v_codes.numel() if not l.protected else 0)
                for l in cache.layers) + 24
    total = idx_bytes + other
    r.update({"sample": f"layer {q[0]} K+V, first {max_tokens} kept tokens of every head",
              "packed_bits_per_symbol": round(8.0 * sum(l.codes.k_codes.numel() + l.codes.v_codes.numel()
                                                        for l in cache.layers if not l.protected) / n_sym_total, 3),
              "cache_ratio_vs_fp16_extrapolated": round(cfg.fp16_bytes / total, 3),
              "bits_per_symbol": round(r["bits_per_symbol"], 4), "delta_seconds": round(r["delta_seconds"], 3),
              "host_seconds": round(r["host_seconds"], 3)})
    rr = E.rans_report(cache, layers=[q[0]], max_tokens=max_tokens)
    r["rans"] = {"container": "encode_e8 (entropy_coder.py:405-452), one stream per (K|V, batch)",
                 "bits_per_symbol": round(rr["bits_per_symbol"], 4), "stream_bytes": rr["stream_bytes"],
                 "device_seconds": round(rr["device_seconds"], 4), "host_seconds": round(rr["host_seconds"], 4),
                 "host_msymbols_per_s": round(rr["host_msymbols_per_s"], 1)}
    c = cache.layers[q[0]].codes
    dev = torch.device("cuda", torch.cuda.current_device())
    st = E.e8_entropy_stats(c.k_codes[:, :, :min(cache.n_kept, max_tokens)].to(dev), cache.head_dim_padded,
                            c.key_levels)
    r["rans"]["shannon_bits_per_symbol_keys"] = round(st["entropy_bps"], 4)  # measure_e8_entropy
    return r


def extras_leg(sh, steps: int) -> dict:
    """Device times of the secondary tensor-core kernels on this step's own data (rank 0, one
    GPU, outside the headline): decode attention over the first quantized layer's codes (8
    query heads per KV head, CUDA-graph replay), and merge eviction's nearest-survivor search on
    unit centroids of 8 value layers, tensor-core screening against the exact fp32 kernel."""
    cfg, dev = sh.cfg, sh.dev
    out = {}
    if sh.quant and cfg.head_dim == 128:
        lc = sh.codes[0]
        b, hl = cfg.batch, sh.hl
        g = torch.Generator(device=dev).manual_seed(0)
        q = (torch.randn(b, 8 * hl, 128, device=dev, generator=g) * 0.3).half()
        outq = torch.empty_like(q)

        def att():
            K.attend_compressed(q, lc, sh.kept_idx, count=sh.kept_count, rope_base=cfg.rope_base,
                                rope_rows=cfg.seq, out=outq)
        att()
        s2 = torch.cuda.Stream()
        s2.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s2):
            att()
        torch.cuda.current_stream().wait_stream(s2)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                att()
        us = timed(graph.replay, 1, 3, 1) / steps * 1e3
        nbytes = sum(t.numel() * t.element_size() for t in (lc.k_codes, lc.v_codes, lc.k_scales, lc.v_scales))
        out["attend_compressed"] = {"us": round(us, 2), "kv_heads": hl, "q_heads": 8 * hl, "tokens": sh.cap,
                                    "gbs_of_compressed_bytes": round(nbytes / us / 1e3, 1),
                                    "kernel": "attend_partial (tcgen05 S = K Q^T, O = C^T W^T) + attend_combine"}
    # the drop-in default layout (fake_quant): codes plus the fp16 reconstruction written back
    fl = sh.quant[:4]
    if fl:
        rk = [torch.empty_like(sh.K[l]) for l in fl]
        rv = [torch.empty_like(sh.V[l]) for l in fl]
        kw = dict(key_levels=sh.levels[0], value_levels=sh.levels[1], kept_idx=sh.kept_idx,
                  kept_count=sh.kept_count, n_kept=sh.cap, rope_base=cfg.rope_base, rope_rows=cfg.seq)
        ms_c = timed(lambda: K.compress_layers([sh.K[l] for l in fl], [sh.V[l] for l in fl], **kw), 5, 3, 1) / 5
        ms_r = timed(lambda: K.compress_layers([sh.K[l] for l in fl], [sh.V[l] for l in fl], recon_k=rk, recon_v=rv,
                                               **kw), 5, 3, 1) / 5
        out["compress_fake_quant"] = {"layers": len(fl), "ms_codes": round(ms_c, 4),
                                      "ms_codes_plus_fp16_reconstruction": round(ms_r, 4)}
        del rk, rv
    layers = sh.quant[:8]
    if cfg.eviction_rate > 0 and len(layers) == 8 and cfg.head_dim == 128 and cfg.batch == 1:
        cen = sum(sh.V[l][0].float().mean(0) for l in layers) / 8.0
        unit = torch.nn.functional.normalize(cen, dim=1).contiguous()
        kept_mask = torch.zeros(cfg.seq, dtype=torch.bool, device=dev)
        kept = sh.kept_idx[0, :int(sh.kept_count[0])].long()
        kept_mask[kept] = True
        ev = torch.nonzero(~kept_mask).flatten()
        res = {}
        for tc in (True, False):
            r = K.merge_nearest(unit, ev, kept, tensor_cores=tc)
            res[tc] = (timed(lambda: K.merge_nearest(unit, ev, kept, tensor_cores=tc), 3, 3, 1) / 3, r)
        out["merge_nearest"] = {"ms_tensor_cores": round(res[True][0], 3), "ms_exact_fp32": round(res[False][0], 3),
                                "evicted": int(ev.numel()), "kept": int(kept.numel()),
                                "same_indices": bool(torch.equal(res[True][1], res[False][1]))}
    return out


# ------------------------------------------------------------------- reference
def run_reference(args, cfg, rank, world):
    if rank != 0:
        return
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, threads, desc = cpu_sample(cfg)
        if i >= args.warmup:
            vals.append(gbs)
    v = sum(vals) / len(vals)
    line = {"metric": METRIC, "impl": "reference", "value": round(v, 4), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, cap_for(cfg), world),
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "cpu": cpu_model(), "sample": desc},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- kernel modes
def run_kernel(args, cfg, dev):
    """--kernel attend|merge: one JSON line timing a compressed-cache kernel outside the
    headline step, on the bench's synthetic layers of the chosen config (1 GPU, CUDA events).

    attend: decode attention over one compressed layer (kernels.attend_compressed) with 8 query
            heads per KV head, against dequantize + torch attention of the same codes.
    merge : merge eviction (kernels.merge_evicted_values) over --merge-layers layers; each
            timed iteration starts from the original values (restored outside the timing)."""
    T, h, d = cfg.seq, cfg.heads, cfg.head_dim
    kl, vl = 2 ** cfg.key_bits, 2 ** cfg.value_bits
    k0, _ = syn.device_layer(cfg, 0, dev)
    imp = K.score_keykey(k0, 32)
    nk = n_keep_for(T, cfg.sliding_window, cfg.eviction_rate)
    idx, cnt = K.select_keep(imp, cfg.sliding_window, nk)
    cap = int(cnt.max())
    line = {"impl": "ours", "n_gpus": 1, "data": "synthetic", "config": {"workload": cfg.name, "seq": T, "heads": h,
                                                                          "head_dim": d, "kept_tokens": cap}}
    if args.kernel == "attend":
        k, v = syn.device_layer(cfg, 3, dev)
        kidx = idx[:, :cap].contiguous()
        lc = K.compress_layers([k], [v], key_levels=kl, value_levels=vl, kept_idx=kidx, kept_count=cnt, n_kept=cap,
                               rope_base=cfg.rope_base)[0]
        del k, v
        hq = 8 * h
        q = (torch.randn(cfg.batch, hq, d, device=dev, generator=torch.Generator(device=dev).manual_seed(0)) * 0.3).half()

        def fused():
            return K.attend_compressed(q, lc, kidx, count=cnt, rope_base=cfg.rope_base, rope_rows=T)

        def unfused():
            ok, ov = K.decompress_layers([lc], kidx, head_dim=d, count=cnt, rope_base=cfg.rope_base, rope_rows=T)
            kk = ok[0][0].float().repeat_interleave(8, 0)
            vv = ov[0][0].float().repeat_interleave(8, 0)
            w = torch.softmax(torch.einsum("hd,hnd->hn", q[0].float(), kk) * d ** -0.5, -1)
            return torch.einsum("hn,hnd->hd", w, vv).half()[None]

        a, b = fused().float(), unfused().float()
        rel = float((a - b).norm() / b.norm())
        fms = timed(fused, args.steps, args.warmup, 1) / args.steps
        ums = timed(unfused, args.steps, args.warmup, 1) / args.steps
        # device time without the Python call path: the same calls captured in a CUDA graph
        gs = torch.cuda.Stream()
        gs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(gs):
            fused()
        torch.cuda.current_stream().wait_stream(gs)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fused()
        gms = timed(graph.replay, 1, args.warmup, 1) / args.steps
        nbytes = sum(t.numel() * t.element_size() for t in (lc.k_codes, lc.v_codes, lc.k_scales, lc.v_scales))
        line.update({"metric": "decode attention over one compressed layer", "value": round(fms * 1e3, 2),
                     "unit": "us", "higher_is_better": False, "q_heads": hq,
                     "device_us_graph": round(gms * 1e3, 2),
                     "compressed_bytes": nbytes, "gbs_of_compressed_bytes": round(nbytes / fms / 1e6, 1),
                     "gbs_of_compressed_bytes_graph": round(nbytes / gms / 1e6, 1),
                     "dequant_then_torch_us": round(ums * 1e3, 2), "rel_l2_vs_dequant_then_torch": rel})
    else:
        L = args.merge_layers
        vs = [syn.device_layer(cfg, l, dev)[1] for l in range(L)]
        backup = [v.clone() for v in vs]
        mask = torch.zeros(cfg.batch, T + 1, dtype=torch.bool, device=dev)
        valid = torch.arange(idx.shape[1], device=dev)[None] < cnt[:, None]
        mask.scatter_(1, torch.where(valid, idx.long(), torch.full_like(idx.long(), T)), True)
        mask = mask[:, :T].contiguous()
        times = []
        for it in range(args.warmup + 5):
            for v, bk in zip(vs, backup):
                v.copy_(bk)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            K.merge_evicted_values(vs, mask, imp)
            e1.record()
            torch.cuda.synchronize()
            if it >= args.warmup:
                times.append(e0.elapsed_time(e1))
        ms = sorted(times)[len(times) // 2]
        n_e = int((~mask).sum())
        fma = n_e * cap * d * cfg.batch
        line.update({"metric": "merge eviction over layers", "value": round(ms, 3), "unit": "ms",
                     "higher_is_better": False, "layers": L, "evicted_tokens": n_e,
                     "similarity_fma": fma, "similarity_tflops_if_all_time": round(2 * fma / ms / 1e9, 1)})
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-per-config", action="store_true", help="skip the configs 1-3 kernel rooflines")
    ap.add_argument("--no-entropy", action="store_true", help="skip the zstd post-step report")
    ap.add_argument("--profile", action="store_true", help="a few steps only (for ncu launch lists)")
    ap.add_argument("--kernel", choices=["attend", "merge"], default=None,
                    help="time one compressed-cache kernel instead of the headline step (1 GPU)")
    ap.add_argument("--merge-layers", type=int, default=8)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    # Native libraries (NCCL's version banner, for one) print to fd 1; the driver reads the one
    # JSON line from stdout, so fd 1 is pointed at stderr and the line goes to the saved stdout.
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = out

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = syn.CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.kernel is not None:
        if rank == 0:
            run_kernel(args, cfg, dev)
        return
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    sh = Shard(cfg, rank, world, dev, group)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    sh.step()  # first call builds the RoPE table cache
    torch.cuda.synchronize()
    sh.launches = 0
    with clocks:
        ms = timed(sh.step, args.steps, args.warmup, world, group)
    launches = sh.launches * args.steps // (args.steps + args.warmup)

    peak, peak_kind = peaks()
    kr = kernel_rooflines(sh, args.steps, peak)
    kms = kr["compress"]["launch_ms"] if kr else float("nan")
    algo = sh.compress_algo_bytes()
    # DRAM bytes (read + write) per algorithmic byte of the compress kernel, from one ncu capture
    # (profiles/traffic.json); traffic of this launch = that ratio x this launch's algorithmic bytes.
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            ratio = json.load(f)["compress_kernel"]["dram_bytes_per_algo_byte"]
        traffic = int(round(ratio * algo)) if sh.quant else None
    except (OSError, KeyError, ValueError):
        pass

    extras = None
    if rank == 0 and world == 1 and not args.profile and not args.no_per_config:
        try:
            extras = extras_leg(sh, args.steps)
        except Exception as ex:  # reported, never fatal: outside the headline
            extras = {"error": f"{type(ex).__name__}: {ex}"}

    e2e, e2e_err, host_cache = None, "disabled", None
    if not args.no_e2e and not args.profile:
        with GpuLocalCpus(local):
            got, e2e_err = e2e_leg(sh, args.e2e_steps)
        if got is not None:
            e2e, host_cache = got
    sh.free()
    torch.cuda.empty_cache()
    ent = None
    if rank == 0 and host_cache is not None and not args.no_entropy:
        try:
            ent = entropy_leg(host_cache, cfg)
        except Exception as ex:  # reported, never fatal: it is outside the measured path
            ent = {"error": f"{type(ex).__name__}: {ex}"}
    per_cfg = None
    if rank == 0 and world == 1 and not args.no_per_config and not args.profile:
        per_cfg = per_config_rooflines(args.config, dev, args.steps, peak)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and not args.profile:
        gbs, threads, desc = cpu_sample(cfg)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
               "sample": desc}

    value = cfg.fp16_bytes * args.steps / (ms / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, sh.cap, world),
            "roofline": {"bound": "hbm", "achieved": kr["compress"]["achieved"] if kr else 0.0, "peak": peak,
                         "unit": "GB/s", "frac": kr["compress"]["frac"] if kr else 0.0,
                         "frac_of_spec_8tbs": round((kr["compress"]["achieved"] if kr else 0.0) / 8000.0, 4),
                         "traffic": traffic, "peak_kind": peak_kind, "kernel": "compress_kernel",
                         "launch_ms": round(kms, 4), "algo_bytes": algo, "units": "rank 0's share"},
            "dequant": ({"value": kr["dequant"]["achieved"], "unit": "GB/s", "frac": kr["dequant"]["frac"],
                         "frac_of_spec_8tbs": round(kr["dequant"]["achieved"] / 8000.0, 4),
                         "launch_ms": kr["dequant"]["launch_ms"], "algo_bytes": algo} if kr else None),
            "per_config": per_cfg,
            "extras": extras,
            "entropy": ent,
            "cpu_baseline": cpu,
            "e2e": e2e if e2e is not None else {"value": None, "unit": "GB/s", "error": e2e_err},
            "gpu_launches": launches,
            "clocks": clocks.report(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
