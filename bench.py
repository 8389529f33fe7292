"""Benchmark of the paged-KV attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--only WORKLOAD] [--no-extras] [--no-cpu-baseline]

Headline (every N, one process per GPU under torchrun): Llama-3-70B-shaped attention
sharded by KV head, the configuration the metric "per GPU at 1/2/4/8 B200" names.
Hq 64, Hkv 8, D 128, bf16, 16-token pages; rank r of N owns KV heads
[r*8/N, (r+1)*8/N) and their Q heads, as its own tensors; no collective on the path.
  * prefill step: reshape_and_cache of 2 x 8192 tokens into a contiguous cache + the
    tcgen05 causal prefill over it.  value = aggregate prefill TFLOP/s of the job
    (algorithmic FLOPs 4*D*Hq*causal pairs over all 64 heads / the slowest rank's
    step time): strong scaling, the total work is fixed.
  * decode step (same line, "decode"): 256 sequences with context U{1024..32768}
    (seed 41), block tables from a random permutation of the page pool (seed 42),
    reshape_and_cache of the 256 new tokens + split-KV decode; aggregate HBM GB/s.
  * e2e: the prefill step through the public torch API with pinned host buffers,
    every step's inputs copied host->device and its output device->host.
  * verify: after timing, each rank's outputs on sampled rows / sequences are
    gathered to rank 0 and checked against a plain torch fp32 attention on the GPU.
Inputs are drawn per head from per-head seeds, so the job computes the same numbers
at every N.

Extras at N=1 (same JSON line): the Llama-3-8B varlen prefill (4 sequences
U{512..2048}, Hq 32, Hkv 8) with its own roofline, its e4m3-cache variant, the
Llama-3-8B decode step (B 64, ctx U{512..8192}, 40k-page pool; unfused, fused, e4m3),
the reshape_and_cache sweep (T in {1, 16, 256, 4096, 65536} x scattered / sequential
x 0 / 10 % padding into a 65,536-page cache), the CPU-runnable fp16 pair (reshape
T 256 + prefill L 256 on the GPU) and rms_norm with the residual add.

Timing: W untimed warm-up steps, then K steps each bracketed by CUDA events on the
launching stream; a step's time is the 10 %-trimmed mean of the K samples (the
reference harness sorts its samples and drops 10 % at each end,
test/src/suite/executor.cpp:270-276); the whole K-step region is bracketed by a
barrier and a device synchronise; multi-GPU times are the max over ranks.  L2 is
flushed (256 MB write) between timed prefill steps; decode and reshape inputs are
larger than L2 unless stated otherwise per key.

--impl reference times the reference's own CPU golden of the path on the host
cores: flash_attn_varlen_func of test/zoo/teco/flash_attention/flash_attention.py
(torch fp32, installed unmodified under baseline/_ref by oracle/install_ref.py), on
a bounded sample of the same workload per step, plus the reshape_and_cache loop
(this repository's C restatement; the reference's is a C++ harness method).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "teco-ops_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

D, BS = 128, 16
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
TRIM = 0.10


# ----------------------------------------------------------------------------- helpers
def cdiv(a, b):
    return (a + b - 1) // b


def causal_pairs(q_lens, kv_lens):
    tot = 0
    for L, S in zip(q_lens, kv_lens):
        for i in range(L):
            tot += max(0, min(S, S - L + i + 1))
    return tot


def attn_flops(q_lens, kv_lens, hq, d=D):
    return 4 * d * hq * causal_pairs(q_lens, kv_lens)


def attn_bytes(q_lens, kv_lens, hq, hkv, d=D, bs=BS, elem=2):
    kv = sum(kv_lens) * hkv * d * elem * 2
    qo = 2 * sum(q_lens) * hq * d * 2
    return kv + qo + 4 * sum(cdiv(s, bs) for s in kv_lens) + 8 * len(q_lens)


def reshape_bytes(n_valid, n_tokens, hkv, d=D):
    return 8 * n_tokens + 4 * n_valid * hkv * d * 2


def trimmed_mean(xs, frac=TRIM):
    s = sorted(xs)
    k = int(len(s) * frac)
    s = s[k:len(s) - k] if len(s) - 2 * k > 0 else s
    return sum(s) / len(s)


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return {k: float(j[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, \
            "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """DRAM bytes per launch from the committed ncu summaries (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every 10 ms while the
    timed regions run (reading only; no setting is changed)."""

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []
        self.smax = None
        self._stop = threading.Event()
        self.t = None

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.dev]) if vis and vis.split(",")[0].isdigit() else self.dev
            self.h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.nv = nv
            self.smax = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # NVML unavailable: report it
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
            except Exception:
                pass
            time.sleep(0.01)

    def stop(self):
        if self.t is None:
            return {"sm_mhz": None, "sm_max_mhz": None,
                    "reasons": ["nvml unavailable: " + getattr(self, "err", "?")]}
        self._stop.set()
        self.t.join(timeout=2)
        nv = self.nv
        names = {nv.nvmlClocksEventReasonHwSlowdown: "hw_slowdown",
                 nv.nvmlClocksEventReasonHwThermalSlowdown: "hw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwThermalSlowdown: "sw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwPowerCap: "sw_power_cap"}
        reasons = set()
        for _, r in self.samples:
            for bit, n in names.items():
                if r & bit:
                    reasons.add(n)
        sm = sorted(c for c, _ in self.samples)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": self.smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def timed_loop(torch, steps, warmup, phases, flush=None):
    """`warmup` untimed iterations, then `steps` iterations of the callables in
    `phases`, each phase bracketed by CUDA events on the current stream; `flush`
    runs between iterations, outside the events.  Returns per-phase lists of ms."""
    for _ in range(warmup):
        for f in phases:
            f()
        if flush:
            flush()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(phases) + 1)]
          for _ in range(steps)]
    for s in range(steps):
        ev[s][0].record()
        for i, f in enumerate(phases):
            f()
            ev[s][i + 1].record()
        if flush:
            flush()
    torch.cuda.synchronize()
    return [[ev[s][i].elapsed_time(ev[s][i + 1]) for s in range(steps)]
            for i in range(len(phases))]


def step_ms(times):
    """Per-step time of a phase list: 10 %-trimmed mean of the summed phases."""
    return trimmed_mean([sum(x) for x in zip(*times)])


class Dist:
    def __init__(self, shard_of=0):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        if self.world > 1:
            dist.init_process_group("nccl", device_id=torch.device("cuda", self.local))
        self.shard_world = shard_of or self.world   # --shard-of: rank 0's shard of an N-way
                                                    # split, alone on one GPU (analysis)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def per_head_randn(torch, lead_shape, heads, seed0, dev, dtype):
    """[*lead_shape[:1], len(heads), *lead_shape[1:]] with head h drawn from seed0 + h
    (the global head index), so a shard holds the same values at every N."""
    out = torch.empty(lead_shape[0], len(heads), *lead_shape[1:], device=dev, dtype=dtype)
    g = torch.Generator(device=dev)
    for i, h in enumerate(heads):
        g.manual_seed(seed0 + h)
        out[:, i] = torch.randn(*lead_shape, device=dev, dtype=dtype, generator=g)
    return out


def torch_attention_rows(torch, q_rows, pos, k, v, group, scale):
    """Plain torch fp32 attention of query rows at positions `pos` (causal: keys
    j <= pos) over keys k / values v [S, Hkv, D]; q_rows [R, Hq, D] -> [R, Hq, D]."""
    qf = q_rows.float().permute(1, 0, 2)                                  # [Hq, R, D]
    kf = k.float().permute(1, 2, 0).repeat_interleave(group, 0)           # [Hq, D, S]
    vf = v.float().permute(1, 0, 2).repeat_interleave(group, 0)           # [Hq, S, D]
    s = torch.matmul(qf, kf) * scale
    j = torch.arange(k.shape[0], device=k.device)
    s = s.masked_fill(j[None, None, :] > pos[None, :, None], float("-inf"))
    return torch.matmul(torch.softmax(s, -1), vf).permute(1, 0, 2)


def err_stats(torch, got, ref):
    d = (got.float() - ref.float()).abs()
    mx, mean = float(d.max()), float(d.mean())
    return {"max_abs": mx, "mean_abs": mean, "ok": bool(mx <= 2e-2 and mean <= 2e-3)}


# ----------------------------------------------------------------------------- headline
class Llama70B:
    """Llama-3-70B-shaped attention sharded by KV head (Hq 64, Hkv 8, D 128, bf16, bs 16)."""

    HQ, HKV, L, NSEQ, B_DEC = 64, 8, 8192, 2, 256
    SEED_Q, SEED_K, SEED_V = 50000, 51000, 52000
    SEED_DK, SEED_DV, SEED_DQ, SEED_NK, SEED_NV = 53000, 54000, 55000, 56000, 57000

    def __init__(self, dd: Dist, with_decode=True):
        import torch
        from tecoops import capi, sharding
        self.torch, self.capi, self.dd = torch, capi, dd
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.shard = s = sharding.head_shard(self.HQ, self.HKV, dd.shard_world,
                                             dd.rank if dd.shard_world == dd.world else 0)
        self.hq, self.hkv = s.q_heads, s.kv_heads
        self.qh = list(range(s.q_begin, s.q_end))
        self.kh = list(range(s.kv_begin, s.kv_end))
        bf = torch.bfloat16
        self.lens = [self.L] * self.NSEQ
        tot = sum(self.lens)
        self.tot = tot
        self.q = per_head_randn(torch, (tot, D), self.qh, self.SEED_Q, dev, bf)
        self.k = per_head_randn(torch, (tot, D), self.kh, self.SEED_K, dev, bf)
        self.v = per_head_randn(torch, (tot, D), self.kh, self.SEED_V, dev, bf)
        pages = [cdiv(n, BS) for n in self.lens]
        self.nb = sum(pages)
        bt = torch.arange(self.nb, dtype=torch.int32).view(self.NSEQ, -1)
        self.bt = bt.to(dev)
        self.slot = torch.arange(tot, device=dev)
        self.kc = torch.zeros(self.nb, self.hkv, BS, D, device=dev, dtype=bf)
        self.vc = torch.zeros_like(self.kc)
        self.qlens = torch.tensor(self.lens, dtype=torch.int32, device=dev)
        self.out = torch.empty_like(self.q)
        self.flops_total = attn_flops(self.lens, self.lens, hq=self.HQ)
        self.flops_local = attn_flops(self.lens, self.lens, hq=self.hq)
        self.h = capi.Handle(torch.cuda.current_stream().cuda_stream)
        self.d = (capi.Desc(capi.DATA_INT32, self.bt.shape),
                  capi.Desc(capi.DATA_BFLOAT16, self.q.shape),
                  capi.Desc(capi.DATA_BFLOAT16, self.kc.shape))
        self.flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)
        if with_decode:
            self._setup_decode()

    def _setup_decode(self):
        torch, capi, dev = self.torch, self.capi, self.dev
        B = self.B_DEC
        ctx = torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(41))
        pages = cdiv(ctx + 1, BS).tolist()
        pool = sum(pages) + 1024
        perm = torch.randperm(pool, generator=torch.Generator().manual_seed(42)).to(torch.int32)
        bt = torch.zeros(B, max(pages), dtype=torch.int32)
        p0 = 0
        for b in range(B):
            bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
            p0 += pages[b]
        bf = torch.bfloat16
        self.dkc = per_head_randn(torch, (pool, BS, D), self.kh, self.SEED_DK, dev, bf)
        self.dvc = per_head_randn(torch, (pool, BS, D), self.kh, self.SEED_DV, dev, bf)
        self.dq = per_head_randn(torch, (B, D), self.qh, self.SEED_DQ, dev, bf)
        self.dknew = per_head_randn(torch, (B, D), self.kh, self.SEED_NK, dev, bf)
        self.dvnew = per_head_randn(torch, (B, D), self.kh, self.SEED_NV, dev, bf)
        slot = [int(bt[b, int(ctx[b]) // BS]) * BS + int(ctx[b]) % BS for b in range(B)]
        self.dslot = torch.tensor(slot, dtype=torch.int64, device=dev)
        self.dctx_h = ctx
        self.dbt_h = bt
        self.dctx = (ctx + 1).to(torch.int32).to(dev)
        self.dones = torch.ones(B, dtype=torch.int32, device=dev)
        self.dbt = bt.to(dev)
        self.dout = torch.empty_like(self.dq)
        self.dd_ = (capi.Desc(capi.DATA_INT32, bt.shape),
                    capi.Desc(capi.DATA_BFLOAT16, self.dq.shape),
                    capi.Desc(capi.DATA_BFLOAT16, self.dkc.shape))
        self.dB, self.dpool, self.dmaxk = B, pool, int(ctx.max()) + 1
        kv = (ctx + 1).tolist()
        self.dbytes_total = attn_bytes([1] * B, kv, hq=self.HQ, hkv=self.HKV) + \
            reshape_bytes(B, B, hkv=self.HKV)
        self.dbytes_local = attn_bytes([1] * B, kv, hq=self.hq, hkv=self.hkv) + \
            reshape_bytes(B, B, hkv=self.hkv)
        self.d_attn_bytes_local = attn_bytes([1] * B, kv, hq=self.hq, hkv=self.hkv)

    def flush(self):
        self.flush_buf.zero_()

    def reshape(self):
        self.capi.check(self.capi.reshape_and_cache(
            self.h, self.k.data_ptr(), self.v.data_ptr(), self.slot.data_ptr(), self.kc.data_ptr(),
            self.vc.data_ptr(), self.tot, self.hkv, D, self.nb, BS), "reshape_and_cache")

    def prefill(self):
        b, q, c = self.d
        self.capi.check(self.capi.flash_attention(
            self.h, self.L, self.L, self.nb, self.qlens.data_ptr(), self.qlens.data_ptr(), b,
            self.bt.data_ptr(), q, self.q.data_ptr(), c, self.kc.data_ptr(), c, self.vc.data_ptr(),
            q, self.out.data_ptr()), "flash_attention prefill")

    def decode_reshape(self):
        self.capi.check(self.capi.reshape_and_cache(
            self.h, self.dknew.data_ptr(), self.dvnew.data_ptr(), self.dslot.data_ptr(),
            self.dkc.data_ptr(), self.dvc.data_ptr(), self.dB, self.hkv, D, self.dpool, BS),
            "reshape_and_cache decode")

    def decode(self):
        b, q, c = self.dd_
        self.capi.check(self.capi.flash_attention(
            self.h, 1, self.dmaxk, self.dpool, self.dones.data_ptr(), self.dctx.data_ptr(), b,
            self.dbt.data_ptr(), q, self.dq.data_ptr(), c, self.dkc.data_ptr(), c,
            self.dvc.data_ptr(), q, self.dout.data_ptr()), "flash_attention decode")

    # ---- verification (outside every timed region)
    def _gather_heads(self, x):
        """[R, Hq/N, D] on every rank -> [R, Hq, D] on every rank (head order)."""
        torch, dd = self.torch, self.dd
        if dd.world == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(dd.world)]
        dd.dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=1)

    def verify(self):
        torch, dev = self.torch, self.dev
        bf = torch.bfloat16
        res = {}
        # prefill: rows at the start, middle and end of each sequence, all 64 heads
        loc = [0, 64, self.L // 2, self.L // 2 + 64, self.L - 64]
        pos = torch.cat([torch.arange(a, a + 64) for a in loc[::2]] +
                        [torch.arange(loc[1], loc[1] + 64)]).to(dev)
        rows = torch.cat([pos + b * self.L for b in range(self.NSEQ)])
        got = self._gather_heads(self.out[rows])
        if self.dd.rank == 0:
            allq, allk = list(range(self.HQ)), list(range(self.HKV))
            q = per_head_randn(torch, (self.tot, D), allq, self.SEED_Q, dev, bf)
            k = per_head_randn(torch, (self.tot, D), allk, self.SEED_K, dev, bf)
            v = per_head_randn(torch, (self.tot, D), allk, self.SEED_V, dev, bf)
            refs = []
            for b in range(self.NSEQ):
                sl = slice(b * self.L, (b + 1) * self.L)
                refs.append(torch_attention_rows(torch, q[sl][pos], pos, k[sl], v[sl],
                                                 self.HQ // self.HKV, D ** -0.5))
            res["prefill"] = dict(err_stats(torch, got, torch.cat(refs)),
                                  rows=int(rows.numel()), heads=self.HQ)
            del q, k, v
        # decode: 8 sampled sequences, all 64 heads
        if hasattr(self, "dq"):
            sample = torch.randperm(self.dB, generator=torch.Generator().manual_seed(44))[:8]
            got = self._gather_heads(self.dout[sample.to(dev)])
            if self.dd.rank == 0:
                allq, allk = list(range(self.HQ)), list(range(self.HKV))
                dq = per_head_randn(torch, (self.dB, D), allq, self.SEED_DQ, dev, bf)
                nk = per_head_randn(torch, (self.dB, D), allk, self.SEED_NK, dev, bf)
                nv = per_head_randn(torch, (self.dB, D), allk, self.SEED_NV, dev, bf)
                ks, vs = [], []
                for h in allk:   # one head's cache at a time, only the sampled pages kept
                    g = torch.Generator(device=dev)
                    kk, vv = [], []
                    for seed, dst in ((self.SEED_DK, kk), (self.SEED_DV, vv)):
                        g.manual_seed(seed + h)
                        full = torch.randn(self.dpool, BS, D, device=dev, dtype=bf, generator=g)
                        for b in sample.tolist():
                            n = int(self.dctx_h[b]) + 1
                            ids = self.dbt_h[b, :cdiv(n, BS)].long().to(dev)
                            dst.append(full[ids].reshape(-1, D)[:n].clone())
                        del full
                    ks.append(kk)
                    vs.append(vv)
                refs = []
                for i, b in enumerate(sample.tolist()):
                    n = int(self.dctx_h[b]) + 1
                    k = torch.stack([ks[h][i] for h in allk], 1)   # [n, Hkv, D]
                    v = torch.stack([vs[h][i] for h in allk], 1)
                    k[n - 1], v[n - 1] = nk[b], nv[b]              # the step's new token
                    refs.append(torch_attention_rows(
                        torch, dq[b:b + 1], torch.tensor([n - 1], device=dev), k, v,
                        self.HQ // self.HKV, D ** -0.5))
                res["decode"] = dict(err_stats(torch, got, torch.cat(refs)),
                                     sequences=len(sample), heads=self.HQ)
        return res


def gpu_local_cpus(torch):
    """CPUs next to the current GPU (NVML's CPU affinity of the device, within this
    process's allowed set), or None when NVML cannot say."""
    try:
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        n = os.cpu_count() or 1
        mask = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
        cpus = {64 * w + b for w, m in enumerate(mask) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:   # no NVML, or no affinity information on this host
        return None


def run_e2e_prefill(W, args, dd):
    """The headline prefill step through the public torch API (tecoops.reshape_and_cache
    + tecoops.flash_attn_varlen_func) with this rank's inputs in pinned host memory:
    every step copies q, the new K/V, slot_mapping, cu_seqlens_q, seqused_k and
    block_table host->device and reads the output back device->host.  Steps are
    pipelined as a serving loop runs them: step i+1's upload (copy stream), step i's
    kernels (compute stream) and step i-1's download (second copy stream) overlap,
    with two sets of device buffers; the timed region spans all K steps, from the first
    upload to the last download, max over ranks."""
    import tecoops
    torch = W.torch
    # the pinned buffers' pages go to the NUMA node of the CPUs that first touch them:
    # run this rank on the CPUs next to its GPU while they are made and used, so that the
    # copies do not cross the socket link (the previous affinity is restored afterwards)
    old_cpus = os.sched_getaffinity(0)
    near = gpu_local_cpus(torch)
    if near:
        os.sched_setaffinity(0, near)
    try:
        res = _e2e_prefill_loop(W, args, dd, tecoops, torch)
    finally:
        os.sched_setaffinity(0, old_cpus)
    res["host_cpus"] = (f"{len(near)} CPUs next to the GPU (NVML affinity)" if near
                        else "unbound (no NVML CPU affinity)")
    return res


def _e2e_prefill_loop(W, args, dd, tecoops, torch):
    host = {n: t.cpu().pin_memory() for n, t in
            (("q", W.q), ("k", W.k), ("v", W.v), ("slot", W.slot), ("bt", W.bt))}
    cu = torch.zeros(len(W.lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(W.lens), 0)
    host["cu"] = cu.pin_memory()
    host["seqused"] = torch.tensor(W.lens, dtype=torch.int32).pin_memory()
    out_h = [torch.empty(W.q.shape, dtype=W.q.dtype).pin_memory() for _ in range(2)]
    dev = [{n: torch.empty_like(t, device="cuda") for n, t in host.items()} for _ in range(2)]
    out_d = [torch.empty_like(W.q) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_h[0].numel() * out_h[0].element_size()
    empty = torch.Tensor()
    s_up, s_comp, s_down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("up", "comp", "down")}
    used = [False, False]

    def step(i):
        b = i % 2
        if used[b]:   # buffer set b is free once step i-2 was computed and downloaded
            s_up.wait_event(ev["comp"][b])
            s_comp.wait_event(ev["down"][b])
        with torch.cuda.stream(s_up):
            for n in host:
                dev[b][n].copy_(host[n], non_blocking=True)
            ev["up"][b].record(s_up)
        s_comp.wait_event(ev["up"][b])
        with torch.cuda.stream(s_comp):
            d = dev[b]
            tecoops.reshape_and_cache(d["k"], d["v"], d["slot"], W.kc, W.vc)
            tecoops.flash_attn_varlen_func(d["q"], W.kc, W.vc, W.L, d["cu"], W.L, empty,
                                           d["seqused"], D ** -0.5, True, empty, d["bt"], False,
                                           out_d[b])
            ev["comp"][b].record(s_comp)
        s_down.wait_event(ev["comp"][b])
        with torch.cuda.stream(s_down):
            out_h[b].copy_(out_d[b], non_blocking=True)
            ev["down"][b].record(s_down)
        used[b] = True

    for i in range(args.warmup):
        step(i)
    dd.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_up)
    for i in range(args.steps):
        step(i)
    t1.record(s_down)
    dd.barrier()
    ms = dd.max(t0.elapsed_time(t1))
    return {"value": args.steps * W.flops_total / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms / args.steps, "h2d_bytes_per_step": h2d * dd.world,
            "d2h_bytes_per_step": d2h * dd.world,
            "per_rank_bytes": {"h2d": h2d, "d2h": d2h},
            "api": "tecoops.reshape_and_cache + tecoops.flash_attn_varlen_func (pinned host "
                   "buffers; upload / kernels / download of consecutive steps overlapped on "
                   "three streams); bytes are the whole job's"}


# ----------------------------------------------------------------------------- extras
class Llama8B:
    """Llama-3-8B-shaped workloads (Hq 32, Hkv 8, D 128, bf16, bs 16) on one GPU."""

    HQ, HKV = 32, 8

    def __init__(self):
        import torch
        from tecoops import capi
        self.torch, self.capi = torch, capi
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(1000)
        bf = torch.bfloat16
        self.lens = torch.randint(512, 2049, (4,), generator=torch.Generator().manual_seed(10)).tolist()
        tot = self.tot = sum(self.lens)
        self.q = torch.randn(tot, self.HQ, D, device=dev, dtype=bf, generator=g)
        self.k = torch.randn(tot, self.HKV, D, device=dev, dtype=bf, generator=g)
        self.v = torch.randn(tot, self.HKV, D, device=dev, dtype=bf, generator=g)
        pages = [cdiv(n, BS) for n in self.lens]
        self.nb = sum(pages)
        bt = torch.zeros(len(self.lens), max(pages), dtype=torch.int32)
        slots, p0 = [], 0
        for b, n in enumerate(self.lens):
            bt[b, :pages[b]] = torch.arange(p0, p0 + pages[b], dtype=torch.int32)
            slots.append(torch.arange(n) + p0 * BS)
            p0 += pages[b]
        self.bt = bt.to(dev)
        self.slot = torch.cat(slots).to(dev)
        self.kc = torch.zeros(self.nb, self.HKV, BS, D, device=dev, dtype=bf)
        self.vc = torch.zeros_like(self.kc)
        self.qlens = torch.tensor(self.lens, dtype=torch.int32, device=dev)
        self.out = torch.empty_like(self.q)
        self.flops = attn_flops(self.lens, self.lens, hq=self.HQ)
        self.h = capi.Handle(torch.cuda.current_stream().cuda_stream)
        self.d_bt = capi.Desc(capi.DATA_INT32, self.bt.shape)
        self.d_q = capi.Desc(capi.DATA_BFLOAT16, self.q.shape)
        self.d_c = capi.Desc(capi.DATA_BFLOAT16, self.kc.shape)
        self.max_q = max(self.lens)
        self.rbytes = reshape_bytes(tot, tot, hkv=self.HKV)
        self.flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)

    def flush(self):
        self.flush_buf.zero_()

    def reshape(self):
        self.capi.check(self.capi.reshape_and_cache(
            self.h, self.k.data_ptr(), self.v.data_ptr(), self.slot.data_ptr(),
            self.kc.data_ptr(), self.vc.data_ptr(), self.tot, self.HKV, D, self.nb, BS),
            "reshape_and_cache")

    def prefill(self):
        self.capi.check(self.capi.flash_attention(
            self.h, self.max_q, self.max_q, self.nb, self.qlens.data_ptr(), self.qlens.data_ptr(),
            self.d_bt, self.bt.data_ptr(), self.d_q, self.q.data_ptr(), self.d_c,
            self.kc.data_ptr(), self.d_c, self.vc.data_ptr(), self.d_q, self.out.data_ptr()),
            "flash_attention")

    # e4m3 cache: reshape_ex quantises, prefill_ex reads it
    def setup_fp8(self):
        torch, capi = self.torch, self.capi
        self.p8_s = 1.0 / 64
        self.p8_kc = torch.zeros(self.kc.shape, dtype=torch.uint8, device=self.dev)
        self.p8_vc = torch.zeros_like(self.p8_kc)
        self.p8_desc = capi.Desc(capi.DATA_FLOAT8_E4M3, self.p8_kc.shape)

    def reshape_fp8(self):
        capi = self.capi
        capi.check(capi.reshape_and_cache_ex(
            self.h, self.k.data_ptr(), self.v.data_ptr(), self.slot.data_ptr(),
            self.p8_kc.data_ptr(), self.p8_vc.data_ptr(), self.tot, self.HKV, D, self.nb, BS,
            capi.DATA_BFLOAT16, cache_dtype=capi.DATA_FLOAT8_E4M3, k_scale=self.p8_s,
            v_scale=self.p8_s), "reshape_and_cache_ex fp8")

    def prefill_fp8(self):
        capi = self.capi
        capi.check(capi.flash_attention_ex(
            self.h, self.max_q, self.max_q, self.nb, self.qlens.data_ptr(), self.qlens.data_ptr(),
            self.d_bt, self.bt.data_ptr(), self.d_q, self.q.data_ptr(), self.p8_desc,
            self.p8_kc.data_ptr(), self.p8_desc, self.p8_vc.data_ptr(), self.d_q,
            self.out.data_ptr(), k_scale=self.p8_s, v_scale=self.p8_s), "flash_attention_ex fp8")

    # decode: B 64, ctx U{512..8192}, 40k-page pool
    def setup_decode(self):
        torch, capi = self.torch, self.capi
        B, pool = 64, 40000
        ctx = torch.randint(512, 8193, (B,), generator=torch.Generator().manual_seed(20))
        perm = torch.randperm(pool, generator=torch.Generator().manual_seed(21)).to(torch.int32)
        pages = cdiv(ctx + 1, BS).tolist()
        bt = torch.zeros(B, max(pages), dtype=torch.int32)
        p0 = 0
        for b in range(B):
            bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
            p0 += pages[b]
        gd = torch.Generator(device=self.dev).manual_seed(2200)
        bf = torch.bfloat16
        self.d_kc = torch.randn(pool, self.HKV, BS, D, device=self.dev, dtype=bf, generator=gd)
        self.d_vc = torch.randn(pool, self.HKV, BS, D, device=self.dev, dtype=bf, generator=gd)
        self.d_q3 = torch.randn(B, self.HQ, D, device=self.dev, dtype=bf, generator=gd)
        self.d_knew = torch.randn(B, self.HKV, D, device=self.dev, dtype=bf, generator=gd)
        self.d_vnew = torch.randn(B, self.HKV, D, device=self.dev, dtype=bf, generator=gd)
        slot = [int(bt[b, int(ctx[b]) // BS]) * BS + int(ctx[b]) % BS for b in range(B)]
        self.d_slot = torch.tensor(slot, dtype=torch.int64, device=self.dev)
        self.d_ctx = (ctx + 1).to(torch.int32).to(self.dev)
        self.d_ones = torch.ones(B, dtype=torch.int32, device=self.dev)
        self.d_bt3 = bt.to(self.dev)
        self.d_out3 = torch.empty_like(self.d_q3)
        self.d_desc = (capi.Desc(capi.DATA_INT32, bt.shape),
                       capi.Desc(capi.DATA_BFLOAT16, self.d_q3.shape),
                       capi.Desc(capi.DATA_BFLOAT16, self.d_kc.shape))
        self.d_B, self.d_pool = B, pool
        self.d_maxk = int(ctx.max()) + 1
        kv = (ctx + 1).tolist()
        self.decode_bytes = attn_bytes([1] * B, kv, hq=self.HQ, hkv=self.HKV)
        self.decode_reshape_bytes = reshape_bytes(B, B, hkv=self.HKV)
        self.f_bytes = attn_bytes([1] * B, kv, hq=self.HQ, hkv=self.HKV, elem=1)
        self.f_reshape_bytes = 8 * B + 2 * B * self.HKV * D * 2 + 2 * B * self.HKV * D

    def decode_reshape(self):
        self.capi.check(self.capi.reshape_and_cache(
            self.h, self.d_knew.data_ptr(), self.d_vnew.data_ptr(), self.d_slot.data_ptr(),
            self.d_kc.data_ptr(), self.d_vc.data_ptr(), self.d_B, self.HKV, D, self.d_pool, BS),
            "reshape_and_cache")

    def decode(self):
        bt_d, q_d, c_d = self.d_desc
        self.capi.check(self.capi.flash_attention(
            self.h, 1, self.d_maxk, self.d_pool, self.d_ones.data_ptr(), self.d_ctx.data_ptr(),
            bt_d, self.d_bt3.data_ptr(), q_d, self.d_q3.data_ptr(), c_d, self.d_kc.data_ptr(),
            c_d, self.d_vc.data_ptr(), q_d, self.d_out3.data_ptr()), "flash_attention")

    def decode_fused(self):
        bt_d, q_d, c_d = self.d_desc
        self.capi.check(self.capi.reshape_and_cache_flash_attention_decode(
            self.h, self.d_knew.data_ptr(), self.d_vnew.data_ptr(), self.d_slot.data_ptr(),
            self.d_maxk, self.d_ones.data_ptr(), self.d_ctx.data_ptr(), bt_d,
            self.d_bt3.data_ptr(), q_d, self.d_q3.data_ptr(), c_d, self.d_kc.data_ptr(), c_d,
            self.d_vc.data_ptr(), q_d, self.d_out3.data_ptr()), "fused decode")

    def setup_decode_fp8(self):
        torch, capi = self.torch, self.capi
        self.f_s = 1.0 / 64
        self.f_kc = (self.d_kc.float() / self.f_s).to(torch.float8_e4m3fn).view(torch.uint8)
        self.f_vc = (self.d_vc.float() / self.f_s).to(torch.float8_e4m3fn).view(torch.uint8)
        self.f_desc = capi.Desc(capi.DATA_FLOAT8_E4M3, self.f_kc.shape)

    def decode_reshape_fp8(self):
        capi = self.capi
        capi.check(capi.reshape_and_cache_ex(
            self.h, self.d_knew.data_ptr(), self.d_vnew.data_ptr(), self.d_slot.data_ptr(),
            self.f_kc.data_ptr(), self.f_vc.data_ptr(), self.d_B, self.HKV, D, self.d_pool, BS,
            capi.DATA_BFLOAT16, cache_dtype=capi.DATA_FLOAT8_E4M3, k_scale=self.f_s,
            v_scale=self.f_s), "reshape_and_cache_ex fp8")

    def decode_fp8(self):
        capi = self.capi
        bt_d, q_d, _ = self.d_desc
        capi.check(capi.flash_attention_ex(
            self.h, 1, self.d_maxk, self.d_pool, self.d_ones.data_ptr(), self.d_ctx.data_ptr(),
            bt_d, self.d_bt3.data_ptr(), q_d, self.d_q3.data_ptr(), self.f_desc,
            self.f_kc.data_ptr(), self.f_desc, self.f_vc.data_ptr(), q_d, self.d_out3.data_ptr(),
            k_scale=self.f_s, v_scale=self.f_s), "flash_attention_ex fp8")


class ReshapeSweep:
    """reshape_and_cache into a 65,536-page bf16 cache (Hkv 8, D 128, bs 16, 2 GiB per
    cache), T new tokens with scattered (random permutation, seed 30) or sequential
    slots and 0 % / 10 % of them -1 (seed 31)."""

    NB, HKV = 65536, 8

    def __init__(self):
        import torch
        from tecoops import capi
        self.torch, self.capi = torch, capi
        dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        bf = torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(3000)
        self.kc = torch.zeros(self.NB, self.HKV, BS, D, device=dev, dtype=bf)
        self.vc = torch.zeros_like(self.kc)
        self.k = torch.randn(65536, self.HKV, D, device=dev, dtype=bf, generator=g)
        self.v = torch.randn(65536, self.HKV, D, device=dev, dtype=bf, generator=g)
        self.perm = torch.randperm(self.NB * BS, generator=torch.Generator().manual_seed(30))
        self.h = capi.Handle(torch.cuda.current_stream().cuda_stream)
        self.flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)

    def slots(self, T, scattered, pad):
        torch = self.torch
        s = self.perm[:T].clone() if scattered else torch.arange(T)
        n_valid = T
        if pad > 0:
            m = torch.rand(T, generator=torch.Generator().manual_seed(31)) < pad
            s[m] = -1
            n_valid = int((~m).sum())
        return s.to(torch.int64).to(self.dev), n_valid

    def run(self, T, slot, steps, warmup):
        def f():
            self.capi.check(self.capi.reshape_and_cache(
                self.h, self.k.data_ptr(), self.v.data_ptr(), slot.data_ptr(), self.kc.data_ptr(),
                self.vc.data_ptr(), T, self.HKV, D, self.NB, BS), "reshape_and_cache")
        # inputs below L2 size are flushed between steps
        fl = (lambda: self.flush_buf.zero_()) if T * self.HKV * D * 2 * 2 < 256e6 else None
        (t,) = timed_loop(self.torch, steps, warmup, [f], flush=fl)
        return trimmed_mean(t)


def cfg1_pair(torch, capi, steps, warmup):
    """The CPU-runnable fp16 pair on the GPU: reshape_and_cache T 256 (H 8, D 128,
    64 pages x 16, slots randperm(1024)[:256] with ~5 % -1) + causal prefill B 1,
    L = S = 256, Hq = Hkv = 8 (the prefill reads K/V from a 16-page region of the
    cache written by reshape)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    f16 = torch.float16
    g = torch.Generator(device=dev).manual_seed(1)
    H, T, NB = 8, 256, 64
    key = torch.randn(T, H, D, device=dev, dtype=f16, generator=g)
    val = torch.randn(T, H, D, device=dev, dtype=f16, generator=g)
    slot = torch.randperm(NB * BS, generator=torch.Generator().manual_seed(2))[:T]
    slot[torch.rand(T, generator=torch.Generator().manual_seed(3)) < 0.05] = -1
    slot = slot.to(torch.int64).to(dev)
    n_valid = int((slot >= 0).sum())
    kc = torch.zeros(NB, H, BS, D, device=dev, dtype=f16)
    vc = torch.zeros_like(kc)
    q = torch.randn(T, H, D, device=dev, dtype=f16, generator=g)
    bt = torch.randperm(NB, generator=torch.Generator().manual_seed(5))[:16].to(torch.int32)
    pslot = (bt.long()[torch.arange(T) // BS] * BS + torch.arange(T) % BS).to(dev)
    bt = bt.view(1, 16).to(dev)
    lens = torch.tensor([T], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    dbt, dq, dc = (capi.Desc(capi.DATA_INT32, bt.shape), capi.Desc(capi.DATA_HALF, q.shape),
                   capi.Desc(capi.DATA_HALF, kc.shape))
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)

    def reshape():
        capi.check(capi.reshape_and_cache(h, key.data_ptr(), val.data_ptr(), slot.data_ptr(),
                                          kc.data_ptr(), vc.data_ptr(), T, H, D, NB, BS), "rc")

    def reshape_p():
        capi.check(capi.reshape_and_cache(h, key.data_ptr(), val.data_ptr(), pslot.data_ptr(),
                                          kc.data_ptr(), vc.data_ptr(), T, H, D, NB, BS), "rc")

    def prefill():
        capi.check(capi.flash_attention(h, T, T, NB, lens.data_ptr(), lens.data_ptr(), dbt,
                                        bt.data_ptr(), dq, q.data_ptr(), dc, kc.data_ptr(), dc,
                                        vc.data_ptr(), dq, out.data_ptr()), "fa")

    tr, = timed_loop(torch, steps, warmup, [reshape], flush=lambda: flush_buf.zero_())
    tp = timed_loop(torch, steps, warmup, [reshape_p, prefill], flush=lambda: flush_buf.zero_())
    fl = attn_flops([T], [T], hq=H)
    return {"workload": "CPU-runnable fp16 pair on the GPU: reshape_and_cache T 256 (H 8, D 128, "
                        "64 x 16 pages, randperm slots, ~5 % -1) and causal prefill B 1, L 256, "
                        "8/8 heads (reshape of its K/V + prefill per step)",
            "reshape_us": trimmed_mean(tr) * 1e3,
            "reshape_gbs": reshape_bytes(n_valid, T, hkv=H) / (trimmed_mean(tr) * 1e-3) / 1e9,
            "prefill_step_us": step_ms(tp) * 1e3,
            "prefill_kernel_us": trimmed_mean(tp[1]) * 1e3,
            "prefill_tflops": fl / (trimmed_mean(tp[1]) * 1e-3) / 1e12,
            "l2": "flushed between steps (inputs < L2); latency-bound at this size",
            "cpu_baseline": cpu_pair(torch, key, val, slot, pslot, q, bt, out, NB, n_valid)}


def cpu_pair(torch, key, val, slot, pslot, q, bt, out_gpu, NB, n_valid):
    """The fp16 pair on the host (same inputs): reshape_and_cache of the 256 tokens (C
    restatement, one thread) and the step of reshape (prefill slots) + the reference
    golden prefill (torch fp32, all host threads); medians of 3 after a warm-up."""
    import numpy as np

    import oracle
    golden = _golden_or_none()
    kw, vw = _words(key), _words(val)
    sl, psl = slot.cpu().numpy(), pslot.cpu().numpy()
    T, H = key.shape[0], key.shape[1]
    kc = np.zeros((NB, H, BS, D), dtype=np.uint16)
    vc = np.zeros_like(kc)
    r_s = _median_s(lambda: oracle.reshape_and_cache(kw, vw, sl, kc, vc))
    res = {"reshape_gbs": reshape_bytes(n_valid, T, hkv=H) / r_s / 1e9, "reshape_cores": 1,
           "kind": "reference"}
    if golden is None:
        return res
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    qf, btc = q.cpu().float(), bt.cpu()
    keep = {}

    def step():
        kc2 = np.zeros((NB, H, BS, D), dtype=np.uint16)
        vc2 = np.zeros_like(kc2)
        oracle.reshape_and_cache(kw, vw, psl, kc2, vc2)
        keep["out"] = golden(qf, _cache_f32(torch, kc2, torch.float16),
                             _cache_f32(torch, vc2, torch.float16), [T], [T], btc)
    p_s = _median_s(step)
    diff = (keep["out"] - out_gpu.cpu().float()).abs()
    res.update({"prefill_step_tflops": attn_flops([T], [T], hq=H) / p_s / 1e12, "cores": threads,
                "sample": f"in full: reshape {r_s * 1e6:.0f} us, reshape + golden prefill "
                          f"{p_s * 1e3:.2f} ms (medians of 3)",
                "gpu_vs_golden": {"max_abs": float(diff.max()), "mean_abs": float(diff.mean())}})
    return res


# ----------------------------------------------------------------------------- CPU arm
def _median_s(fn, runs=3, warmup=1):
    """Wall-clock median of `runs` calls of fn after `warmup` calls."""
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(runs):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return sorted(ts)[len(ts) // 2]


def _words(t):
    """A CUDA or CPU 16-bit tensor as a host numpy array of uint16 words."""
    import numpy as np
    return t.contiguous().cpu().view(__import__("torch").int16).numpy().view(np.uint16)


def _cache_f32(torch, words, dtype):
    """The golden's input conversion (python_api_test/test_flash_attention.py:167-181):
    16-bit cache words [NB, H, bs, D] -> fp32 [NB, bs, H, D]."""
    return (torch.from_numpy(words.view("int16")).view(dtype).float().permute(0, 2, 1, 3)
            .contiguous())


def _cpu_result(value, unit, sample, threads, extra=None):
    r = {"value": value, "unit": unit, "cores": threads, "kind": "reference", "sample": sample}
    if extra:
        r.update(extra)
    return r


def cpu_llama8b_prefill(W, golden):
    """The whole Llama-3-8B prefill step on the host cores: reshape_and_cache of all tokens
    (C restatement of the reference loop, one thread) and the reference golden over the
    batch (torch fp32, all host threads); median of 3 after a warm-up.  Also compares the
    GPU output of the same inputs with the golden's."""
    import numpy as np
    import torch

    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    kw, vw, slot = _words(W.k), _words(W.v), W.slot.cpu().numpy()
    q = W.q.cpu().float()
    bt = W.bt.cpu()
    res = {}

    def step():
        kc = np.zeros((W.nb, W.HKV, BS, D), dtype=np.uint16)
        vc = np.zeros_like(kc)
        oracle.reshape_and_cache(kw, vw, slot, kc, vc)
        res["out"] = golden(q, _cache_f32(torch, kc, torch.bfloat16),
                            _cache_f32(torch, vc, torch.bfloat16), W.lens, W.lens, bt)
    secs = _median_s(step)
    diff = (res["out"] - W.out.cpu().float()).abs()
    return _cpu_result(W.flops / secs / 1e12, "TFLOP/s",
                       f"the whole step (reshape_and_cache of {W.tot} tokens + the golden "
                       f"flash_attn_varlen_func over the {len(W.lens)} sequences), median of 3: "
                       f"{secs:.2f} s",
                       threads, {"gpu_vs_golden": {"max_abs": float(diff.max()),
                                                   "mean_abs": float(diff.mean())}})


def cpu_llama8b_decode(W, golden, out_gpu):
    """The Llama-3-8B decode step on the host cores: reshape_and_cache of the 64 new tokens
    (C loop) and the golden for every sequence on its own pages (the cache compacted per
    sequence, block table remapped to 0..n-1: the golden's math unchanged, its fp32
    conversion limited to the pages the sequence reads); median of 3."""
    import numpy as np
    import torch

    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    kc, vc = _words(W.d_kc), _words(W.d_vc)     # the pool (2 x 1.3 GB), copied untimed
    kw, vw, slot = _words(W.d_knew), _words(W.d_vnew), W.d_slot.cpu().numpy()
    q = W.d_q3.cpu().float()
    ctx = W.d_ctx.cpu().tolist()
    bt = W.d_bt3.cpu().numpy()
    outs = [None] * W.d_B

    def step():
        oracle.reshape_and_cache(kw, vw, slot, kc, vc)
        for b in range(W.d_B):
            pages = bt[b, :cdiv(ctx[b], BS)]
            outs[b] = golden(q[b:b + 1], _cache_f32(torch, kc[pages], torch.bfloat16),
                             _cache_f32(torch, vc[pages], torch.bfloat16), [1], [ctx[b]],
                             torch.arange(len(pages), dtype=torch.int32)[None])
    secs = _median_s(step, runs=3, warmup=0)
    diff = (torch.cat(outs) - out_gpu.cpu().float()).abs()
    step_bytes = W.decode_bytes + W.decode_reshape_bytes
    return _cpu_result(step_bytes / secs / 1e9, "GB/s",
                       f"the whole step (reshape_and_cache of {W.d_B} tokens + the golden per "
                       f"sequence on its compacted pages), median of 3: {secs:.2f} s", threads,
                       {"gpu_vs_golden": {"max_abs": float(diff.max()),
                                          "mean_abs": float(diff.mean())}})


def cpu_reshape_sweep(R, points):
    """Every point of the reshape sweep on the host: the C restatement of the reference
    loop, one thread as the reference runs it, into host caches of the same 65,536 pages
    (touched before timing); median of 3 (2 at T = 65,536)."""
    import numpy as np
    kw, vw = _words(R.k), _words(R.v)
    kc = np.ones((R.NB, R.HKV, BS, D), dtype=np.uint16)
    vc = np.ones_like(kc)
    import oracle
    for pt in points:
        T = pt["T"]
        slot, nv = R.slots(T, pt["slots"] == "scattered", pt["pad"])
        sl = slot.cpu().numpy()
        secs = _median_s(lambda: oracle.reshape_and_cache(kw[:T], vw[:T], sl, kc, vc),
                         runs=2 if T >= 65536 else 3)
        pt["cpu_gbs"] = pt["bytes"] / secs / 1e9
    return {"unit": "GB/s", "cores": 1, "kind": "reference",
            "sample": "every point in full (the C restatement of reshape_and_cache.cpp:136-147, "
                      "one thread), median of 3 (2 at T = 65,536): cpu_gbs of each point"}


def _ref_golden():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import install_ref
    return install_ref.load_golden()


def cpu_sample_70b(golden, b_idx, kv_head, rows=2048, threads=None):
    """One bounded sample of the headline prefill on the host: the reference golden
    (torch fp32) for the last `rows` query rows of one 8192-token sequence and the 8 Q
    heads of one KV head (a chunked prefill of `rows` rows over 8192 keys, which the
    golden handles natively), preceded by reshape_and_cache of that head's 8192 tokens
    with the C restatement of the reference loop.  Returns (algorithmic flops, s)."""
    import numpy as np
    import torch

    import oracle
    if threads:
        torch.set_num_threads(threads)
    L, g = Llama70B.L, Llama70B.HQ // Llama70B.HKV
    gen = torch.Generator().manual_seed(7000 + 16 * b_idx + kv_head)
    q = torch.randn(rows, g, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(L, 1, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(L, 1, D, generator=gen).to(torch.bfloat16)
    nb = cdiv(L, BS)
    kc = np.zeros((nb, 1, BS, D), dtype=np.uint16)
    vc = np.zeros_like(kc)
    kw = k.view(torch.int16).numpy().view(np.uint16)
    vw = v.view(torch.int16).numpy().view(np.uint16)
    slot = np.arange(L, dtype=np.int64)
    bt = torch.arange(nb, dtype=torch.int32)[None]
    t0 = time.perf_counter()
    oracle.reshape_and_cache(kw, vw, slot, kc, vc)
    # the golden's input conversion (python_api_test/test_flash_attention.py:167-181):
    # 16-bit -> fp32, cache [NB, H, bs, D] -> [NB, bs, H, D]
    kf = torch.from_numpy(kc.view(np.int16)).view(torch.bfloat16).float().permute(0, 2, 1, 3)
    vf = torch.from_numpy(vc.view(np.int16)).view(torch.bfloat16).float().permute(0, 2, 1, 3)
    golden(q.float(), kf.contiguous(), vf.contiguous(), [rows], [L], bt)
    return attn_flops([rows], [L], hq=g), time.perf_counter() - t0


def _golden_or_none():
    try:
        return _ref_golden()
    except ImportError:
        return None


def cpu_baseline_70b(budget_s=15.0):
    """Reported CPU baseline of the headline: as many bounded samples as fit in
    ~budget_s (at least one), the reference golden if installed, else not reported."""
    try:
        golden = _ref_golden()
    except ImportError as e:
        return {"value": None, "unavailable": str(e)}
    import torch
    threads = os.cpu_count() or 1
    flops, secs, n = 0, 0.0, 0
    cpu_sample_70b(golden, 0, 0, threads=threads)   # warm-up (allocator, thread pool)
    while n == 0 or secs < budget_s:
        f, t = cpu_sample_70b(golden, n % 2, n % 8, threads=threads)
        flops, secs, n = flops + f, secs + t, n + 1
        if n >= 16:
            break
    return {"value": flops / secs / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "reference",
            "sample": f"{n} samples of the headline prefill, each the last 2048 query rows of "
                      "one 8192-token sequence x the 8 Q heads of one KV head over all 8192 keys "
                      "(the reference golden flash_attn_varlen_func, torch fp32, from "
                      "baseline/_ref; reshape_and_cache of that head's 8192 tokens by the C "
                      f"restatement of the reference loop): {secs:.1f} s on the host"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return   # under torchrun only rank 0 times the CPU path
    world = int(os.environ.get("WORLD_SIZE", "1"))
    try:
        golden = _ref_golden()
    except ImportError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference golden not "
                          f"installed ({e})"}), flush=True)
        return
    import torch
    threads = os.cpu_count() or 1
    flops, secs = 0, 0.0
    for s in range(args.warmup + args.steps):
        f, t = cpu_sample_70b(golden, s % 2, s % 8, threads=threads)
        if s >= args.warmup:
            flops, secs = flops + f, secs + t
    value = flops / secs / 1e12
    line = {
        "impl": "reference", "metric": "prefill TFLOP/s", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (reference CPU golden)", "data": "synthetic",
        "config": {"workload": "Llama-3-70B-shaped causal prefill (Hq 64, Hkv 8, D 128, 2 x 8192 "
                               "tokens, reshape_and_cache + attention); each step a bounded "
                               "sample of it", "same_config": True},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "reference",
                         "sample": "each step: the last 2048 query rows of one 8192-token "
                                   "sequence x the 8 Q heads of one KV head over all 8192 keys, "
                                   "through the reference's own golden flash_attn_varlen_func "
                                   "(test/zoo/teco/flash_attention/flash_attention.py:79-140, "
                                   "torch fp32, unmodified copy in baseline/_ref), after "
                                   "reshape_and_cache of that head's tokens (C restatement of "
                                   "the reference loop, reshape_and_cache.cpp:136-147)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- our arm
def run_extras(args, peaks, torch):
    """Single-GPU extra keys of the N=1 line."""
    ex = {}
    W = Llama8B()
    tr, tp = timed_loop(torch, args.steps, args.warmup, [W.reshape, W.prefill], flush=W.flush)
    k_ms = trimmed_mean(tp)
    traffic = load_traffic().get("fa_prefill_tcgen05_sm100/llama8b")
    ex["llama8b_prefill"] = {
        "workload": "Llama-3-8B varlen causal prefill, 4 seqs L~U{512..2048} "
                    f"({'+'.join(map(str, W.lens))} tokens), Hq 32, Hkv 8, D 128, bs 16, bf16; "
                    "step = reshape_and_cache of all tokens + prefill",
        "metric": "prefill TFLOP/s", "unit": "TFLOP/s",
        "value": W.flops / (step_ms([tr, tp]) * 1e-3) / 1e12,
        "ms_per_step": step_ms([tr, tp]),
        "reshape_us": trimmed_mean(tr) * 1e3,
        "reshape_gbs": W.rbytes / (trimmed_mean(tr) * 1e-3) / 1e9,
        "roofline": {"bound": "tensor", "kernel": "fa_prefill_tcgen05_sm100",
                     "achieved": W.flops / (k_ms * 1e-3) / 1e12, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": W.flops / (k_ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
                     "kernel_us": k_ms * 1e3, "flops_per_launch": W.flops,
                     "traffic": traffic, "peak_source": "bf16_tflops (burst)"},
        "l2": "flushed between timed steps (256 MB write)"}
    golden = _golden_or_none()
    if golden is not None:
        ex["llama8b_prefill"]["cpu_baseline"] = cpu_llama8b_prefill(W, golden)
    W.setup_fp8()
    fr, fp = timed_loop(torch, args.steps, args.warmup, [W.reshape_fp8, W.prefill_fp8],
                        flush=W.flush)
    ex["llama8b_prefill"]["fp8_cache"] = {
        "api": "tecoopsReshapeAndCacheEx + tecoopsFlashAttentionEx, e4m3 cache (scale 1/64)",
        "value": W.flops / (step_ms([fr, fp]) * 1e-3) / 1e12, "ms_per_step": step_ms([fr, fp]),
        "prefill_us": trimmed_mean(fp) * 1e3}
    W.setup_decode()
    tr, ta = timed_loop(torch, args.steps, args.warmup, [W.decode_reshape, W.decode])
    out_bf16 = W.d_out3.clone()
    (tf,) = timed_loop(torch, args.steps, args.warmup, [W.decode_fused])
    W.setup_decode_fp8()
    fr, fa = timed_loop(torch, args.steps, args.warmup, [W.decode_reshape_fp8, W.decode_fp8])
    a_ms, s_ms = trimmed_mean(ta), step_ms([tr, ta])
    step_bytes = W.decode_bytes + W.decode_reshape_bytes
    ex["llama8b_decode"] = {
        "workload": "Llama-3-8B paged decode: B 64, ctx U{512..8192}+1, 40k-page pool, bs 16, "
                    "bf16; step = reshape_and_cache of the 64 new tokens + split-KV decode",
        "metric": "decode HBM GB/s", "unit": "GB/s",
        "value": step_bytes / (s_ms * 1e-3) / 1e9, "ms_per_step": s_ms,
        "attn_kernel_us": a_ms * 1e3,
        "attn_frac_of_measured_hbm": W.decode_bytes / (a_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
        "fused": {"api": "tecoopsReshapeAndCacheFlashAttentionDecode (one launch + merge)",
                  "ms_per_step": trimmed_mean(tf),
                  "value": step_bytes / (trimmed_mean(tf) * 1e-3) / 1e9},
        "fp8_cache": {"api": "tecoopsReshapeAndCacheEx + tecoopsFlashAttentionEx, e4m3 cache",
                      "ms_per_step": step_ms([fr, fa]),
                      "attn_kernel_us": trimmed_mean(fa) * 1e3,
                      "attn_frac_of_measured_hbm": W.f_bytes / (trimmed_mean(fa) * 1e-3) / 1e9
                      / peaks["hbm_gbs"],
                      "speedup_vs_bf16_step": s_ms / step_ms([fr, fa])},
        "l2": "inputs (1.1 GB of K/V) larger than L2"}
    if golden is not None:
        ex["llama8b_decode"]["cpu_baseline"] = cpu_llama8b_decode(W, golden, out_bf16)
    del W
    torch.cuda.empty_cache()
    R = ReshapeSweep()
    sweep = []
    for T in (1, 16, 256, 4096, 65536):
        for scattered in (True, False):
            for pad in (0.0, 0.1):
                slot, nv = R.slots(T, scattered, pad)
                ms = R.run(T, slot, args.steps, args.warmup)
                by = reshape_bytes(nv, T, hkv=R.HKV)
                sweep.append({"T": T, "slots": "scattered" if scattered else "sequential",
                              "pad": pad, "us": ms * 1e3, "bytes": by,
                              "gbs": by / (ms * 1e-3) / 1e9,
                              "frac_of_measured_hbm": by / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]})
    ex["reshape_sweep"] = {
        "workload": "reshape_and_cache into a 65,536-page bf16 cache (Hkv 8, D 128, bs 16, 2 GiB "
                    "per cache); bytes 8*T + 4*valid*Hkv*D*2; L2 flushed between steps when the "
                    "inputs are below 256 MB",
        "metric": "reshape_and_cache HBM GB/s", "unit": "GB/s", "points": sweep}
    ex["reshape_sweep"]["cpu_baseline"] = cpu_reshape_sweep(R, sweep)
    del R
    torch.cuda.empty_cache()
    from tecoops import capi
    ex["fp16_pair"] = cfg1_pair(torch, capi, args.steps, args.warmup)
    ex["rms_norm"] = run_rms(args, peaks, torch)
    return ex


def run_rms(args, peaks, torch):
    from tecoops import capi
    dev = torch.device("cuda", torch.cuda.current_device())
    nT, hidden = 97056, 4096
    g = torch.Generator(device=dev).manual_seed(4000)
    bf = torch.bfloat16
    x = torch.randn(nT, hidden, device=dev, dtype=bf, generator=g)
    r = torch.randn(nT, hidden, device=dev, dtype=bf, generator=g)
    w = torch.randn(hidden, device=dev, dtype=bf, generator=g)
    y, ro = torch.empty_like(x), torch.empty_like(x)
    nbytes = nT * hidden * 2 * 4 + hidden * 2
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)

    def f():
        capi.check(capi.rms_norm(h, x.data_ptr(), w.data_ptr(), r.data_ptr(), y.data_ptr(),
                                 ro.data_ptr(), nT, hidden, 1e-6, dtype=capi.DATA_BFLOAT16), "rms")
    (t,) = timed_loop(torch, args.steps, args.warmup, [f])
    ms = trimmed_mean(t)
    return {"workload": f"rms_norm with residual add, {nT} tokens x hidden 4096, bf16",
            "metric": "rms_norm HBM GB/s", "unit": "GB/s", "value": nbytes / (ms * 1e-3) / 1e9,
            "kernel_us": ms * 1e3, "frac_of_measured_hbm": nbytes / (ms * 1e-3) / 1e9
            / peaks["hbm_gbs"], "l2": f"inputs ({nbytes / 1e6:.0f} MB) larger than L2"}


def run_shard_of(args):
    """Rank 0's share of an N-way KV-head split of the headline, alone on one GPU (no
    process group): the per-rank prefill and decode kernel times that bound the N-GPU
    step, for analysing the scaling curve without holding N GPUs."""
    dd = Dist(shard_of=args.shard_of)
    import torch
    W = Llama70B(dd)
    tr, tp = timed_loop(torch, args.steps, args.warmup, [W.reshape, W.prefill], flush=W.flush)
    td, ta = timed_loop(torch, args.steps, args.warmup, [W.decode_reshape, W.decode])
    print(json.dumps({"shard_of": args.shard_of, "kv_heads": W.hkv, "q_heads": W.hq,
                      "prefill_step_ms": step_ms([tr, tp]), "prefill_kernel_us": trimmed_mean(tp) * 1e3,
                      "reshape_us": trimmed_mean(tr) * 1e3,
                      "prefill_tflops_per_gpu": W.flops_local / (trimmed_mean(tp) * 1e-3) / 1e12,
                      "decode_step_ms": step_ms([td, ta]), "decode_kernel_us": trimmed_mean(ta) * 1e3,
                      "decode_gbs_per_gpu": W.d_attn_bytes_local / (trimmed_mean(ta) * 1e-3) / 1e9}))


def run_ours(args):
    if args.shard_of:
        run_shard_of(args)
        return
    dd = Dist()
    import torch
    peaks, peak_src = load_peaks()
    if args.only:
        run_only(args, dd, torch)
        dd.close()
        return
    W = Llama70B(dd)
    clocks = ClockSampler(dd.local)
    dd.barrier()
    clocks.start()
    # ---- headline: prefill step (reshape + prefill) of this rank's heads
    tr, tp = timed_loop(torch, args.steps, args.warmup, [W.reshape, W.prefill], flush=W.flush)
    dd.barrier()
    ms = dd.max(step_ms([tr, tp]))
    k_ms = trimmed_mean(tp)
    value = W.flops_total / (ms * 1e-3) / 1e12
    achieved = W.flops_local / (k_ms * 1e-3) / 1e12
    k_ms_max = dd.max(k_ms)
    # ---- decode step of the same shards
    td, ta = timed_loop(torch, args.steps, args.warmup, [W.decode_reshape, W.decode])
    dd.barrier()
    dms = dd.max(step_ms([td, ta]))
    da_ms = trimmed_mean(ta)
    clk = clocks.stop()
    e2e = run_e2e_prefill(W, args, dd)
    verify = W.verify()
    del W.dkc, W.dvc
    torch.cuda.empty_cache()
    extras = {}
    if dd.world == 1 and not args.no_extras:
        clocks2 = ClockSampler(dd.local)
        clocks2.start()
        extras = run_extras(args, peaks, torch)
        extras["clocks"] = clocks2.stop()
    cpu = None
    if dd.rank == 0 and dd.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_70b(budget_s=args.cpu_budget)
    if dd.rank == 0:
        # DRAM bytes of one launch from the committed N=1 ncu capture, scaled by this
        # rank's share of the heads (traffic is proportional to the heads a rank holds)
        t1 = load_traffic().get("fa_prefill_tcgen05_sm100/llama70b_n1")
        traffic = t1 * W.flops_local / W.flops_total if t1 else None
        line = {
            "metric": "prefill TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": dd.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) Q/K/V per head, Llama-3-70B head shapes)",
            "config": {"workload": "Llama-3-70B-shaped attention sharded by KV head: Hq 64, Hkv 8, "
                                   "D 128, bf16, bs 16; prefill step = reshape_and_cache of "
                                   "2 x 8192 tokens + causal prefill",
                       "seq_lens": W.lens,
                       "parallelism": f"KV heads split over {dd.world} GPU(s): "
                                      f"{W.hkv} KV / {W.hq} Q heads per rank, no collective",
                       "l2": "flushed between timed prefill steps (256 MB write)",
                       "timing": "per-step CUDA events, 10 %-trimmed mean of K steps, max over "
                                 "ranks"},
            "gpu_launches": 2 * args.steps,
            "roofline": {"bound": "tensor", "kernel": "fa_prefill_tcgen05_sm100",
                         "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"],
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         "traffic": traffic, "flops_per_launch": W.flops_local,
                         "kernel_us": k_ms * 1e3, "kernel_us_max_over_ranks": k_ms_max * 1e3},
            "reshape_us_per_step": trimmed_mean(tr) * 1e3,
            "decode": {"workload": "Llama-3-70B-shaped paged decode sharded by KV head: B 256, "
                                   "ctx U{1024..32768}+1, bs 16, random block tables; step = "
                                   "reshape_and_cache of the 256 new tokens + split-KV decode",
                       "metric": "decode HBM GB/s", "unit": "GB/s",
                       "value": W.dbytes_total / (dms * 1e-3) / 1e9, "ms_per_step": dms,
                       "attn_kernel_us": da_ms * 1e3,
                       "per_gpu_attn_frac_of_measured_hbm":
                           W.d_attn_bytes_local / (da_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                       "l2": f"inputs ({W.dbytes_local / 1e9:.1f} GB per GPU) larger than L2"},
            "e2e": e2e,
            "verify": verify,
            "clocks": clk,
        }
        line.update(extras)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    dd.close()


def run_only(args, dd, torch):
    """One workload's timed loop only (profiler captures run this)."""
    if args.only in ("prefill70b", "decode70b"):
        W = Llama70B(dd, with_decode=args.only == "decode70b")
        ph, fl = ([W.reshape, W.prefill], W.flush) if args.only == "prefill70b" else \
            ([W.decode_reshape, W.decode], None)
    elif args.only in ("prefill8b", "prefill8b_fp8"):
        W = Llama8B()
        if args.only == "prefill8b":
            ph, fl = [W.reshape, W.prefill], W.flush
        else:
            W.setup_fp8()
            ph, fl = [W.reshape_fp8, W.prefill_fp8], W.flush
    elif args.only in ("decode8b", "decode8b_fp8"):
        W = Llama8B()
        W.setup_decode()
        ph, fl = [W.decode_reshape, W.decode], None
        if args.only == "decode8b_fp8":
            W.setup_decode_fp8()
            ph = [W.decode_reshape_fp8, W.decode_fp8]
    elif args.only == "rms_norm":
        print(json.dumps({"only": "rms_norm", **run_rms(args, load_peaks()[0], torch)}))
        return
    elif args.only.startswith("reshape"):
        R = ReshapeSweep()
        T = int(args.only[len("reshape"):] or 65536)
        slot, _ = R.slots(T, True, 0.0)
        print(json.dumps({"only": args.only, "us": R.run(T, slot, args.steps, args.warmup) * 1e3}))
        return
    else:
        raise SystemExit(f"unknown --only {args.only}")
    t = timed_loop(torch, args.steps, args.warmup, ph, flush=fl)
    print(json.dumps({"only": args.only, "ms_per_phase": [trimmed_mean(x) for x in t]}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--shard-of", type=int, default=0,
                    help="analysis: time rank 0's shard of an N-way KV-head split on one GPU")
    ap.add_argument("--only", default=None,
                    help="one workload's timed loop (prefill70b, decode70b, prefill8b, "
                         "prefill8b_fp8, decode8b, decode8b_fp8, rms_norm, reshape<T>)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
