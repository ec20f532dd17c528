"""Decode-attention benchmark: KV-read TB/s and us per decode step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--windows R]
                    [--impl ours|reference] [--workload config2|...|sweep]

One step = one decode call over one batch: every sequence's K/V is read once.
N=1 workload: config 2 (fp16 varlen + sinks, B=32, QH=32, KVH=8, D=128, lens
U[8192,16384] seed 0; 1.545 GB of KV, larger than L2, so no flush is needed).
N>1 (torchrun, one process per GPU, NCCL): weak scaling -- rank r decodes its
own config-2 batch drawn with seed r; no collective on the data path.

``value`` is whole-job KV bytes / device time per step (TB/s): R windows
(default 50) of exactly K back-to-back steps, each bracketed by a barrier and
a device synchronisation on both sides and timed with CUDA events; the
window time is the max over ranks and the median window is reported
(``spread`` gives min / p90 / max).  ``isolated_us_per_call`` (=
``roofline.kernel_us``) is the decode kernel's own duration per call from
events the library records around each launch.  ``e2e`` is the same metric
through the public API with the per-step inputs (q and the sequence lengths)
copied from pinned host memory and the output copied back inside the timed
region; the KV cache is resident on the GPU, as in a serving engine.
``strong`` (every N, unless --no-strong) is the multi-GPU configuration of
the benchmark plan, config 5 (B=128 e4m3 paged + sinks, log-U lengths to
131072) sharded across the ranks by greedy LPT: max-over-ranks us per step,
aggregate TB/s, speed-up against the whole batch on one GPU, and the output
all-gather over NCCL timed once, outside the timed windows.

``--impl reference`` times the reference's own CPU implementation of the
path, its torch ``ref_attention`` (unmodified, installed in baseline/_ref)
on all host threads over the whole batch per step; ``--workload sweep``
reproduces the reference's published sweeps with its Triton kernel timed
beside this library on the same GPU.
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

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from fasterkernels_b200 import workloads as W  # noqa: E402

METRIC = "decode-attn KV-read TB/s"
UNIT = "TB/s"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML
    polled from a thread every ~2 ms (read-only queries).  A decode step is a
    fraction of a millisecond, so the timed windows are repeated (50 by
    default) to give the sampler a region long enough to see."""
    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.sm, self.mask = [], 0
        self.max_mhz = None
        self.th = None
        self.stop_flag = False
        self.err = None

    def _poll(self, nv, h):
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag:
            try:
                self.sm.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                self.mask |= int(get_reasons(h))
            except Exception as e:  # pragma: no cover
                self.err = repr(e)
                return
            time.sleep(0.002)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.idx]) if vis and vis.split(",")[self.idx].isdigit() else self.idx
            h = nv.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.nv = nv
            self.th = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.th.start()
        except Exception as e:
            self.err = repr(e)

    def stop(self):
        self.stop_flag = True
        if self.th is not None:
            self.th.join(timeout=2)
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [f"no samples ({self.err})"]}
        reasons = sorted(n for n, attr in self.REASONS.items() if self.mask & int(getattr(self.nv, attr, 0)))
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.sm), "source": "NVML, 2 ms"}


# ---------------------------------------------------------------- workloads
def setup_workload(name, rank, world, device):
    """Build this rank's share of the workload on `device`.  Returns a dict
    with a zero-arg `run()` (one decode step through the public API), the
    per-step inputs for the e2e leg, algorithmic KV bytes and a config dict."""
    import fasterkernels_b200 as fk
    if name in ("config2", "config2s", "config2g16", "config2d64"):
        # config2g16 / config2d64: config 2's lengths with a 16-head GQA group
        # (128 query heads) / with head dim 64 (64 query heads), shapes the
        # reference's Triton kernels take beyond the benchmark configs
        spec = W.CONFIGS[2]
        lens = W.config_lengths(2, seed=0)
        if name == "config2s":  # profiling case: first 8 sequences (~0.4 GB of KV, still > L2)
            lens = lens[:8]
        qh = {"config2g16": 128, "config2d64": 64}.get(name, spec.q_heads)
        hd = 64 if name == "config2d64" else 128
        d = W.make_varlen(lens, qh, spec.kv_heads, torch.float16, device, seed=rank, sinks=True, head_dim=hd)
        q, k, v, cu, s = d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"]
        out = torch.empty_like(q)

        def run(qq=q, cc=cu, oo=out):
            return fk.flash_decode_gqa_varlen(qq, k, v, cc, s, out=oo)
        kvb = W.kv_bytes(lens, spec.kv_heads, 2, hd)
        suffix = {"config2": "", "config2s": "_first8", "config2g16": "_g16", "config2d64": "_d64"}[name]
        cfg = {"workload": spec.name + suffix, "batch_per_gpu": len(lens),
               "global_batch": len(lens) * world,
               "q_heads": qh, "kv_heads": spec.kv_heads, "head_dim": hd,
               "seq_lens": "U[8192,16384] seed 0 (same per-GPU work on every rank; q/k/v/s_aux seed = rank)", "tokens_this_rank": int(sum(lens)),
               "kv_layout": "contiguous varlen [T, KV_H, D] fp16", "sinks": True,
               "l2": "inputs larger than L2 (>=0.77 GB KV per GPU, no flush)",
               "parallelism": f"dp{world} (each rank its own batch, no collective)"}
        return dict(run=run, q=q, lens_dev=cu, out=out, kv_bytes=kvb, cfg=cfg, scaling="weak",
                    sample=(q, k, v, cu, s, lens), dtype="fp16 in / fp32 accumulate")
    if name == "config3v":  # config-3 lengths in the contiguous varlen layout (comparison / profiling)
        spec = W.CONFIGS[3]
        lens = W.config_lengths(3, seed=0)
        d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, device, seed=rank, sinks=False)
        q, k, v, cu = d["q"], d["k"], d["v"], d["cu_seqlens"]
        out = torch.empty_like(q)

        def run(qq=q, cc=cu, oo=out):
            return fk.flash_decode_gqa_varlen(qq, k, v, cc, out=oo)
        cfg = {"workload": spec.name + "_as_varlen", "batch_per_gpu": spec.batch, "global_batch": spec.batch * world,
               "q_heads": spec.q_heads, "kv_heads": spec.kv_heads, "head_dim": 128,
               "seq_lens": "U[512,8192] seed 0 (same on every rank; data seed = rank)", "kv_layout": "contiguous varlen fp16", "sinks": False,
               "l2": "inputs larger than L2", "parallelism": f"dp{world} (each rank its own batch)"}
        return dict(run=run, q=q, lens_dev=cu, out=out, kv_bytes=W.kv_bytes(lens, spec.kv_heads, 2), cfg=cfg,
                    scaling="weak", sample=None, dtype="fp16 in / fp32 accumulate")
    if name == "config3":
        spec = W.CONFIGS[3]
        lens = W.config_lengths(3, seed=0)
        d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, device, seed=rank, sinks=False)
        kp, vp, bt = W.varlen_to_paged(d["k"], d["v"], lens, spec.pool_factor, seed=rank)
        del d["k"], d["v"]
        q = d["q"]
        sl = torch.tensor(lens, dtype=torch.int32, device=device)
        out = torch.empty_like(q)

        def run(qq=q, ll=sl, oo=out):
            return fk.paged_flash_decode(qq, kp, vp, bt, ll, 16, out=oo)
        cfg = {"workload": spec.name, "batch_per_gpu": spec.batch, "global_batch": spec.batch * world,
               "q_heads": spec.q_heads, "kv_heads": spec.kv_heads, "head_dim": 128,
               "seq_lens": "U[512,8192] seed 0 (same on every rank; data seed = rank)", "pool_pages": int(kp.shape[0]),
               "kv_layout": "paged 16-token pages (random permutation of a x1.25 pool), fp16", "sinks": False,
               "l2": "inputs larger than L2", "parallelism": f"dp{world} (each rank its own batch)"}
        return dict(run=run, q=q, lens_dev=sl, out=out, kv_bytes=W.kv_bytes(lens, spec.kv_heads, 2), cfg=cfg,
                    scaling="weak", sample=None, dtype="fp16 in / fp32 accumulate")
    if name == "config4d":  # config 4 on the HF dense BHSD cache (flash_decode_gqa_hf_fp8 path)
        spec = W.CONFIGS[4]
        lens = W.config_lengths(4, seed=0)
        B, S = spec.batch, lens[0]
        d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, device, seed=rank, sinks=True)
        k8, sk = W.quantize_e4m3(d["k"])
        del d["k"]
        v8, sv = W.quantize_e4m3(d["v"])
        del d["v"]
        kc = k8.view(B, S, spec.kv_heads, 128).transpose(1, 2).contiguous()
        vc = v8.view(B, S, spec.kv_heads, 128).transpose(1, 2).contiguous()
        del k8, v8
        q, s = d["q"], d["s_aux"]
        cl = torch.tensor(lens, dtype=torch.int32, device=device)
        out = torch.empty_like(q)

        def run(qq=q, ll=cl, oo=out):
            return fk.flash_decode_gqa_hf_fp8(qq, kc, vc, ll, None, sk, sv, torch.float16, s_aux=s, out=oo)
        cfg = {"workload": spec.name + "_hf_dense", "batch_per_gpu": B, "global_batch": B * world,
               "q_heads": spec.q_heads, "kv_heads": spec.kv_heads, "head_dim": 128, "seq_lens": "32768 all",
               "kv_layout": "HF dense [B, KV_H, S, D] e4m3 KV (per-tensor scale), fp16 Q", "sinks": True,
               "l2": "inputs larger than L2", "parallelism": f"dp{world} (each rank its own batch)"}
        return dict(run=run, q=q, lens_dev=cl, out=out, kv_bytes=W.kv_bytes(lens, spec.kv_heads, 1), cfg=cfg,
                    scaling="weak", sample=None, dtype="e4m3 KV / fp16 Q / fp32 accumulate")
    if name == "config4":
        spec = W.CONFIGS[4]
        lens = W.config_lengths(4, seed=0)
        d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, device, seed=rank, sinks=True)
        k8, sk = W.quantize_e4m3(d["k"])
        del d["k"]
        v8, sv = W.quantize_e4m3(d["v"])
        del d["v"]
        kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.0, seed=rank)
        del k8, v8
        kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
        q, s = d["q"], d["s_aux"]
        sl = torch.tensor(lens, dtype=torch.int32, device=device)
        out = torch.empty_like(q)

        def run(qq=q, ll=sl, oo=out):
            return fk.paged_flash_decode(qq, kp, vp, bt, ll, 16, s_aux=s, scale_k=sk, scale_v=sv, out=oo)
        cfg = {"workload": spec.name, "batch_per_gpu": spec.batch, "global_batch": spec.batch * world,
               "q_heads": spec.q_heads, "kv_heads": spec.kv_heads, "head_dim": 128, "seq_lens": "32768 all",
               "kv_layout": "paged 16-token pages, e4m3 KV (per-tensor scale amax/448), fp16 Q", "sinks": True,
               "l2": "inputs larger than L2", "parallelism": f"dp{world} (each rank its own batch)"}
        return dict(run=run, q=q, lens_dev=sl, out=out, kv_bytes=W.kv_bytes(lens, spec.kv_heads, 1), cfg=cfg,
                    scaling="weak", sample=None, dtype="e4m3 KV / fp16 Q / fp32 accumulate")
    if name == "config5":
        spec = W.CONFIGS[5]
        all_lens = W.config_lengths(5, seed=0)
        mine = W.lpt_partition(all_lens, world)[rank]
        lens = [all_lens[i] for i in mine]
        # KV drawn in fp16 on the device, then quantised per tensor to e4m3
        d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, device, seed=rank, sinks=True)
        k8, sk = W.quantize_e4m3(d["k"])
        del d["k"]
        v8, sv = W.quantize_e4m3(d["v"])
        del d["v"]
        kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=rank)
        del k8, v8
        kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
        q, s = d["q"], d["s_aux"]
        sl = torch.tensor(lens, dtype=torch.int32, device=device)
        out = torch.empty_like(q)

        def run(qq=q, ll=sl, oo=out):
            return fk.paged_flash_decode(qq, kp, vp, bt, ll, 16, s_aux=s, scale_k=sk, scale_v=sv, out=oo)
        kvb = W.kv_bytes(lens, spec.kv_heads, 1)
        cfg = {"workload": spec.name, "global_batch": spec.batch, "batch_this_rank": len(lens),
               "q_heads": spec.q_heads, "kv_heads": spec.kv_heads, "head_dim": 128,
               "seq_lens": "logU[4096,131072] seed 0, LPT-sharded by KV bytes",
               "kv_layout": "paged 16-token pages, e4m3 KV, fp16 Q", "sinks": True,
               "l2": "inputs larger than L2", "parallelism": f"sequence-sharded x{world}, no collective"}
        return dict(run=run, q=q, lens_dev=sl, out=out, kv_bytes=kvb, cfg=cfg, scaling="strong",
                    sample=None, dtype="e4m3 KV / fp16 Q / fp32 accumulate", indices=mine, batch=spec.batch)
    raise SystemExit(f"unknown workload {name}")




# ---------------------------------------------------------------- timing helpers
def time_steps(fn, steps, stream):
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    ev1.synchronize()
    return ev0.elapsed_time(ev1)


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_vec(xs, world, device, op="max"):
    if world == 1:
        return list(xs)
    import torch.distributed as dist
    t = torch.tensor(list(xs), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def timed_windows(fn, steps, windows, stream, world, device):
    """`windows` timed regions of exactly `steps` back-to-back calls, each
    bracketed by a barrier and a device synchronisation on both sides; the
    per-window time is the max over ranks.  Returns per-window ms."""
    per = []
    for _ in range(windows):
        barrier(world)
        torch.cuda.synchronize()
        per.append(time_steps(fn, steps, stream))
        torch.cuda.synchronize()
        barrier(world)
    return reduce_vec(per, world, device, "max")


def spread(ms_windows, steps):
    us = sorted(m / steps * 1e3 for m in ms_windows)
    n = len(us)
    return {"windows": n, "median_us": round(statistics.median(us), 2), "min_us": round(us[0], 2),
            "p90_us": round(us[min(n - 1, int(0.9 * n))], 2), "max_us": round(us[-1], 2)}


def isolated_kernel_us(run, calls):
    """Mean duration of the decode kernel, from events the library records on
    the launching stream right before and after each launch."""
    from fasterkernels_b200 import _native as N
    torch.cuda.synchronize()
    N.profile_begin(calls)
    for _ in range(calls):
        run()
    ms, n = N.profile_end()
    return ms / max(n, 1) * 1e3


# ---------------------------------------------------------------- our arm
def measure_strong(args, rank, world, local_rank, device):
    """Config 5 (B=128 e4m3 paged + sinks, lens log-U[4096,131072]) sharded
    across the ranks by greedy LPT over KV bytes: max-over-ranks us per step,
    aggregate TB/s, and the speed-up against the whole batch on one GPU (rank
    0 alone, measured in the same run).  The output all-gather over NCCL is
    timed once, outside the timed windows."""
    from fasterkernels_b200 import _native as N
    from fasterkernels_b200.shard import gather_outputs
    stream = torch.cuda.current_stream(device)
    wl = setup_workload("config5", rank, world, device)
    for _ in range(max(args.warmup, 3)):
        wl["run"]()
    wins = timed_windows(wl["run"], args.steps, max(args.windows // 5, 5), stream, world, device)
    ms_step = statistics.median(wins) / args.steps
    tot_bytes = reduce_vec([float(wl["kv_bytes"])], world, device, "sum")[0]
    rec = {"workload": "config5_paged_e4m3_sinks_longctx", "scaling": "strong",
           "parallelism": f"sequence-sharded x{world} (greedy LPT over KV bytes), no collective",
           "us_per_step": round(ms_step * 1e3, 2), "value": round(tot_bytes / (ms_step * 1e-3) / 1e12, 4),
           "unit": UNIT, "kv_bytes_total": int(tot_bytes), "spread": spread(wins, args.steps),
           "isolated_kernel_us_rank0": round(isolated_kernel_us(wl["run"], args.steps), 2)}
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        gather_outputs(wl["out"], wl["indices"], wl["batch"])  # warm-up (first use of all_gather)
        torch.cuda.synchronize()
        dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        full = gather_outputs(wl["out"], wl["indices"], wl["batch"])
        t1.record(stream)
        t1.synchronize()
        g_ms = reduce_vec([t0.elapsed_time(t1)], world, device, "max")[0]
        rec["gather_outputs_us"] = round(g_ms * 1e3, 1)
        rec["gather_bytes"] = int(full.numel() * full.element_size())
        del full
    if N.read_status(device) != 0:
        raise SystemExit("device status word set during the config-5 run")
    del wl
    torch.cuda.empty_cache()
    if world > 1:
        # the same batch on one GPU (rank 0 alone) for the speed-up
        barrier(world)
        if rank == 0:
            one = setup_workload("config5", 0, 1, device)
            for _ in range(max(args.warmup, 3)):
                one["run"]()
            w1 = timed_windows(one["run"], args.steps, max(args.windows // 5, 5), stream, 1, device)
            one_ms = statistics.median(w1) / args.steps
            rec["one_gpu_us_per_step"] = round(one_ms * 1e3, 2)
            rec["speedup_vs_1gpu"] = round(one_ms / ms_step, 3)
            del one
            torch.cuda.empty_cache()
        barrier(world)
    else:
        rec["one_gpu_us_per_step"] = rec["us_per_step"]
        rec["speedup_vs_1gpu"] = 1.0
    return rec


def reference_cpu_leg(workload, seqs, min_seconds, config1):
    """Run the reference arm in a child process (it imports the reference's
    own module, which must not share this GPU process) and parse its line."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", workload,
           "--steps", "1", "--warmup", "1", "--ref-seqs", str(seqs), "--ref-min-seconds", str(min_seconds)]
    if config1:
        cmd.append("--ref-config1")
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        return {"error": r.stderr.strip().splitlines()[-1:] or ["failed"]}
    return json.loads(r.stdout.strip().splitlines()[-1])


def run_ours(args, rank, world, local_rank):
    from fasterkernels_b200 import _native as N
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    wl = setup_workload(args.workload, rank, world, device)
    cfg, dtype, scaling = wl["cfg"], wl["dtype"], wl["scaling"]
    stream = torch.cuda.current_stream(device)
    for _ in range(max(args.warmup, 3)):
        wl["run"]()
    torch.cuda.synchronize()
    if N.read_status(device) != 0:
        raise SystemExit("device status word set during warm-up")

    # ---- headline: `windows` x K back-to-back steps, inputs resident in HBM
    clocks = ClockSampler(local_rank)
    clocks.start()
    wins = timed_windows(wl["run"], args.steps, args.windows, stream, world, device)
    clk = clocks.stop()
    ms_step = statistics.median(wins) / args.steps
    tot_bytes = reduce_vec([float(wl["kv_bytes"])], world, device, "sum")[0]
    value = tot_bytes / (ms_step * 1e-3) / 1e12

    # ---- the decode kernel's own duration per call (library events on the
    # launching stream right before and after each launch)
    kern_us = isolated_kernel_us(wl["run"], args.steps)
    rank_bytes = float(wl["kv_bytes"])

    # ---- e2e: pinned host q + lengths in, output back, every step.  Serial:
    # copy in, decode, copy out on one stream.  Pipelined (the headline e2e):
    # as a serving loop runs it, step i+1's inputs are copied in on an H2D
    # stream while step i decodes and step i-1's output is copied out on a
    # D2H stream (two buffer sets; events order every reuse).  Both include
    # all K steps' copies inside the timed region.
    q_h = wl["q"].cpu().pin_memory()
    l_h = wl["lens_dev"].cpu().pin_memory()
    o_h = [torch.empty(wl["out"].shape, dtype=wl["out"].dtype).pin_memory() for _ in range(2)]

    def e2e_step():
        wl["q"].copy_(q_h, non_blocking=True)
        wl["lens_dev"].copy_(l_h, non_blocking=True)
        wl["run"]()
        o_h[0].copy_(wl["out"], non_blocking=True)
    for _ in range(3):
        e2e_step()
    es_wins = timed_windows(e2e_step, args.steps, max(args.windows // 5, 5), stream, world, device)
    e_serial = statistics.median(es_wins) / args.steps

    qd = [wl["q"], wl["q"].clone()]
    ld = [wl["lens_dev"], wl["lens_dev"].clone()]
    od = [wl["out"], torch.empty_like(wl["out"])]
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def e2e_window(steps):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        in_ok = [torch.cuda.Event() for _ in range(2)]   # inputs of buffer b landed
        k_done = [torch.cuda.Event() for _ in range(2)]  # decode of buffer b finished
        out_ok = [torch.cuda.Event() for _ in range(2)]  # output of buffer b copied out
        ev0.record(stream)
        h2d_s.wait_event(ev0)
        d2h_s.wait_event(ev0)

        def copy_in(i):
            b = i & 1
            with torch.cuda.stream(h2d_s):
                if i >= 2:
                    h2d_s.wait_event(k_done[b])
                qd[b].copy_(q_h, non_blocking=True)
                ld[b].copy_(l_h, non_blocking=True)
                in_ok[b].record(h2d_s)
        copy_in(0)
        for i in range(steps):
            b = i & 1
            if i + 1 < steps:
                copy_in(i + 1)
            stream.wait_event(in_ok[b])
            if i >= 2:
                stream.wait_event(out_ok[b])
            wl["run"](qd[b], ld[b], od[b])
            k_done[b].record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(k_done[b])
                o_h[b].copy_(od[b], non_blocking=True)
                out_ok[b].record(d2h_s)
        stream.wait_stream(h2d_s)
        stream.wait_stream(d2h_s)
        ev1.record(stream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)
    e2e_window(3)
    e_wins = []
    for _ in range(max(args.windows // 5, 5)):
        barrier(world)
        torch.cuda.synchronize()
        e_wins.append(e2e_window(args.steps))
        torch.cuda.synchronize()
        barrier(world)
    e_wins = reduce_vec(e_wins, world, device, "max")
    e_step = statistics.median(e_wins) / args.steps
    h2d = q_h.numel() * q_h.element_size() + l_h.numel() * l_h.element_size()
    d2h = o_h[0].numel() * o_h[0].element_size()
    if N.read_status(device) != 0:
        raise SystemExit("device status word set during the timed region")
    sample = wl["sample"]
    del wl, q_h, l_h, o_h, qd, ld, od
    torch.cuda.empty_cache()

    strong = None
    if not args.no_strong and args.workload != "config5":
        strong = measure_strong(args, rank, world, local_rank, device)

    if rank != 0:
        return None
    peak, peak_kind = load_peaks()
    achieved = rank_bytes / (kern_us * 1e-6) / 1e9  # rank 0's bytes over rank 0's kernel time
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            tr = json.load(f).get(args.workload)
            if tr:
                traffic = tr["bytes_per_launch"]
    except Exception:
        pass
    rec = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "us_per_step": round(ms_step * 1e3, 2),
        "isolated_us_per_call": round(kern_us, 2), "spread": spread(wins, args.steps),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded N(0,1) q/k/v/s_aux; no dataset)", "config": cfg,
        "roofline": {"bound": "hbm", "kernel": "decode_split_kernel", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s", "traffic": traffic, "kernel_us": round(kern_us, 2),
                     "bytes_per_launch": int(rank_bytes)},
        "e2e": {"value": round(tot_bytes / (e_step * 1e-3) / 1e12, 4), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e_step, 5),
                "serial_value": round(tot_bytes / (e_serial * 1e-3) / 1e12, 4),
                "serial_ms_per_step": round(e_serial, 5),
                "note": "public API; every step copies q and the lengths in from pinned host memory and its "
                        "output back; copies of step i+1 / i-1 overlap step i's decode on H2D / D2H streams "
                        "(serial_*: all on one stream); KV resident"},
        "gpu_launches": args.steps * args.windows,
        "clocks": clk,
    }
    if strong is not None:
        rec["strong"] = strong
    if world == 1 and sample is not None and not args.no_cpu_baseline:
        leg = reference_cpu_leg(args.workload, seqs=4, min_seconds=10.0, config1=True)
        if "error" in leg:
            rec["cpu_baseline"] = {"value": None, "unit": UNIT, "error": leg["error"]}
        else:
            cb = dict(leg["cpu_baseline"])
            cb["value"] = leg["value"]
            rec["cpu_baseline"] = cb
            if "config1_full" in leg:
                rec["cpu_config1_full"] = leg["config1_full"]
    return rec


# ---------------------------------------------------------------- reference arm
def load_reference_ref_attention():
    """The reference's own CPU implementation of this path, its torch
    ``ref_attention`` (fskernels/tilelang/tilelang_gqa_decode.py:174-207),
    from the unmodified install in baseline/_ref.  Returns (fn, why_not)."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "fskernels")):
        return None, "baseline/_ref not installed"
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from fskernels.tilelang.tilelang_gqa_decode import ref_attention
        return ref_attention, None
    except Exception as e:  # pragma: no cover
        return None, f"import failed: {e!r}"[:200]


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path on all host threads:
    its torch ``ref_attention`` in fp32 (from baseline/_ref; the numpy
    restatement in oracle/ if that install is missing), called per sequence
    as the reference's varlen tests loop (tests/test_triton_fd_gqa.py:68-141).
    Rank 0 only.  By default every timed step is the WHOLE workload batch."""
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    ref_fn, why = load_reference_ref_attention()
    if args.workload in ("config3", "config3v", "config4", "config4d", "config5"):
        spec = W.CONFIGS[int(args.workload[6])]
        lens = W.config_lengths(spec, seed=0)
        kvh, qh, es = spec.kv_heads, spec.q_heads, (1 if spec.kv_dtype == torch.float8_e4m3fn else 2)
    else:
        spec = W.CONFIGS[2]
        lens = W.config_lengths(2, seed=0)
        kvh, qh, es = spec.kv_heads, {"config2g16": 128, "config2d64": 64}.get(args.workload, spec.q_heads), 2
    hd = 64 if args.workload == "config2d64" else 128
    n = len(lens) if args.ref_seqs <= 0 else min(args.ref_seqs, len(lens))
    sel = lens[:n]
    d = W.make_varlen(sel, qh, kvh, torch.float16, "cpu", seed=0, sinks=True, head_dim=hd)
    cu = d["cu_seqlens"].tolist()
    # per-sequence fp32 operands in the reference's layout [1, KV_H, L, D]
    seqs = [(d["q"][b:b + 1].float(), d["k"][cu[b]:cu[b + 1]].float().transpose(0, 1).unsqueeze(0).contiguous(),
             d["v"][cu[b]:cu[b + 1]].float().transpose(0, 1).unsqueeze(0).contiguous(),
             torch.tensor([sel[b]])) for b in range(n)]
    sink = d["s_aux"]
    qn, kn, vn = d["q"].float().numpy(), d["k"].numpy(), d["v"].numpy()

    def step():
        if ref_fn is not None:
            for q, k, v, L in seqs:
                ref_fn(q, k, v, L, qh, sink)
        else:
            from oracle import gqa_decode_oracle as O
            O.decode_varlen(qn, kn, vn, np.asarray(cu), sink.numpy(), dtype=np.float32)

    byt = W.kv_bytes(sel, kvh, es, hd)
    for _ in range(args.warmup):
        step()
    reps, t0 = 0, time.perf_counter()
    while True:
        step()
        reps += 1
        el = time.perf_counter() - t0
        if reps >= args.steps and el >= args.ref_min_seconds:
            break
    val = byt * reps / el / 1e12
    kind = "reference" if ref_fn is not None else "port"
    impl = ("fskernels ref_attention (torch fp32, baseline/_ref)" if ref_fn is not None
            else f"numpy fp32 restatement in oracle/ ({why})")
    whole = n == len(lens)
    desc = (f"{'the whole batch' if whole else f'first {n} of {len(lens)} sequences'} "
            f"({sum(sel)} tokens, KV_H={kvh}) per step, {impl}, {torch.get_num_threads()} threads")
    cores = torch.get_num_threads() if ref_fn is not None else (os.cpu_count() or 1)
    rec = {"impl": "reference", "metric": METRIC, "value": round(val, 6), "unit": UNIT, "n_gpus": world,
           "steps": reps, "warmup": args.warmup, "ms_per_step": round(el / reps * 1e3, 3),
           "higher_is_better": True, "scaling": "strong" if args.workload == "config5" else "weak",
           "vs_baseline": None, "dtype": "fp32 (CPU)", "data": "synthetic",
           "config": {"workload": spec.name + {"config2g16": "_g16", "config2d64": "_d64"}.get(args.workload, ""),
                      "same_config": whole, "sample": desc},
           "cpu_baseline": {"value": round(val, 6), "unit": UNIT, "cores": cores, "kind": kind, "sample": desc},
           "e2e": {"value": round(val, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.ref_config1:
        rec["config1_full"] = time_config1(ref_fn)
    return rec


def time_config1(ref_fn):
    """Config 1 timed in full (B=4, Q_H=32, KV_H=8, D=128, lens U[1,2048]
    seed 0, sinks, fp32) with the reference's ref_attention on the padded
    batch, exactly its call signature."""
    spec = W.CONFIGS[1]
    lens = W.config_lengths(1, seed=0)
    d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float32, "cpu", seed=0, sinks=True)
    S = max(lens)
    k = torch.zeros(len(lens), spec.kv_heads, S, 128)
    v = torch.zeros_like(k)
    cu = d["cu_seqlens"].tolist()
    for b, L in enumerate(lens):
        k[b, :, :L] = d["k"][cu[b]:cu[b + 1]].transpose(0, 1)
        v[b, :, :L] = d["v"][cu[b]:cu[b + 1]].transpose(0, 1)
    kl = torch.tensor(lens)
    if ref_fn is None:
        return {"error": "reference not installed"}
    ref_fn(d["q"], k, v, kl, spec.q_heads, d["s_aux"])
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 5.0:
        ref_fn(d["q"], k, v, kl, spec.q_heads, d["s_aux"])
        reps += 1
    el = (time.perf_counter() - t0) / reps
    return {"workload": spec.name, "lens": lens, "ms_per_call": round(el * 1e3, 3), "calls": reps,
            "kv_bytes_fp32": W.kv_bytes(lens, spec.kv_heads, 4), "threads": torch.get_num_threads()}


# ---------------------------------------------------------------- sweep
def run_sweep(args):
    """The reference's published sweeps (benchmarks/benchmark.py:82-116,155-158):
    max S in {512..32768} at B=4 and B in {1..32} at max S=16384, fp16,
    Q_H=32, KV_H=8, D=128, lens randint(max(64, S/4), S+1) seed 42, sinks
    randn*0.1.  Per point: this library through its Python entry point
    (triton.testing.do_bench, as the reference times, which flushes L2
    between calls), its kernel alone (library events), and the reference's
    Triton kernel K1 from baseline/_ref, JIT-compiled for this GPU, through
    its own entry point under the same do_bench."""
    import fasterkernels_b200 as fk
    from triton.testing import do_bench
    dev = torch.device("cuda", 0)
    path = os.path.join(ROOT, "baseline", "_ref")
    k1, k1_why = None, None
    if args.sweep_no_ref:
        k1_why = "not requested (--sweep-no-ref)"
    elif os.path.isdir(os.path.join(path, "fskernels")):
        sys.path.insert(0, path)
        try:
            from fskernels.triton.triton_gqa_decode import flash_decode_gqa_varlen as k1
        except Exception as e:  # pragma: no cover
            k1_why = repr(e)[:200]
    else:
        k1_why = "baseline/_ref not installed"
    pts = [("S", s, 4, s) for s in (512, 1024, 2048, 4096, 8192, 16384, 32768)] + \
          [("B", b, b, 16384) for b in (1, 2, 4, 8, 16, 32)]
    out = []
    for kind, param, B, S in pts:
        torch.manual_seed(42)
        kl = torch.randint(max(64, S // 4), S + 1, size=(B,), device=dev)
        cu = torch.zeros(B + 1, device=dev, dtype=torch.int32)
        cu[1:] = torch.cumsum(kl, 0).to(torch.int32)
        T = int(cu[-1])
        q = torch.randn(B, 32, 128, device=dev, dtype=torch.float16)
        k = torch.randn(T, 8, 128, device=dev, dtype=torch.float16)
        v = torch.randn(T, 8, 128, device=dev, dtype=torch.float16)
        sink = torch.randn(32, device=dev) * 0.1
        o = torch.empty_like(q)
        ours = lambda: fk.flash_decode_gqa_varlen(q, k, v, cu, sink, out=o)  # noqa: E731
        for _ in range(5):
            ours()
        t_ours = do_bench(ours, warmup=25, rep=200) * 1e3
        kern = isolated_kernel_us(ours, 50)
        row = {"sweep": kind, "param": param, "batch": B, "max_s": S, "tokens": T,
               "kv_bytes": T * 8 * 128 * 2 * 2, "ours_entry_us": round(t_ours, 2), "ours_kernel_us": round(kern, 2)}
        if k1 is not None:
            try:
                for _ in range(3):
                    k1(q, k, v, cu, sink)
                row["ref_triton_k1_entry_us"] = round(do_bench(lambda: k1(q, k, v, cu, sink), warmup=25, rep=200)
                                                      * 1e3, 2)
                row["speedup_vs_k1"] = round(row["ref_triton_k1_entry_us"] / t_ours, 2)
            except Exception as e:  # pragma: no cover
                row["ref_triton_k1_error"] = repr(e)[:200]
        out.append(row)
        del q, k, v
    return {"metric": "decode-attn us per call (reference sweep protocol)", "unit": "us", "n_gpus": 1,
            "higher_is_better": False, "data": "synthetic (benchmark.py's setup_inputs protocol, seed 42)",
            "dtype": "fp16", "ref_triton_k1": "timed" if k1 is not None else f"unavailable: {k1_why}",
            "points": out}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--windows", type=int, default=50, help="timed windows of K steps (median reported)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["config2", "config2s", "config2g16", "config2d64", "config3", "config3v",
                                           "config4", "config4d", "config5", "sweep"], default="config2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong", action="store_true", help="skip the config-5 strong-scaling record")
    ap.add_argument("--ref-seqs", type=int, default=0, help="reference arm: sequences per step (0 = all)")
    ap.add_argument("--ref-min-seconds", type=float, default=0.0, help="reference arm: keep timing until this long")
    ap.add_argument("--ref-config1", action="store_true", help="reference arm: also time config 1 in full")
    ap.add_argument("--sweep-no-ref", action="store_true", help="sweep: skip the reference's Triton kernel")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload == "sweep":
            args.workload = "config2"
        rec = run_reference(args, rank, world)
    elif args.workload == "sweep":
        rec = run_sweep(args) if rank == 0 else None
    else:
        if world > 1:
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        rec = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rec is not None:
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
