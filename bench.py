"""Benchmark: batch-1 greedy decode of the Qwen2.5-3B-shaped int4 model.

Workload: synthetic N(0, 0.02) weights quantised
by the reference quantiser (int4 g128 layers with f32 scales, int8-row tied
LM head), 32-token uniform-random prompt, greedy decode at ctx ~128: each
"step" is one decoded token; positions cycle through 32..159 so the context
stays ~128 however many steps are timed.  `--ctx 4096` runs configs[2]
(prefill 4096, decode at ctx 4096..4160).

Arms:
  (default)          the CUDA library: CUDA-event time on the runtime's stream
                     of K chained decode steps, all inputs resident in HBM.
  --impl reference   the reference's CPU path (the C restatement in oracle/)
                     on all host cores, same metric, bounded sample.

Multi-GPU (torchrun): replicas only -- every rank decodes its own request
stream with its own copy of the weights; no data-path collective.  value =
tokens of all ranks / max-over-ranks device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s @ctx 128/4096; int4 GEMV achieved HBM GB/s vs peak"
SEED = 0xE6B00000
PROMPT_SEED = 0xE6B00010
N_PROMPT = 32


def cfg_bytes(cfg, kv_f16=True):
    """Algorithmic bytes of one decode token: every weight byte read once
    (int4 layers + f32 group scales + q/k/v bias + norms, int8 LM head + f32
    row scales) + the KV cache read at ctx (bytes per position)."""
    H, I, L, V = cfg["hiddenSize"], cfg["intermediateSize"], cfg["numLayers"], cfg["vocabSize"]
    QD = cfg["numHeads"] * cfg["headDim"]
    KVD = cfg["numKVHeads"] * cfg["headDim"]
    per_layer_w = (QD + 2 * KVD) * H // 2 + H * QD // 2 + 2 * I * H // 2 + H * I // 2
    per_layer_s = ((QD + 2 * KVD) * H + H * QD + 2 * I * H + H * I) // 128 * 4
    per_layer_small = (QD + 2 * KVD) * 4 + 2 * H * 4
    weights = L * (per_layer_w + per_layer_s + per_layer_small) + V * H + V * 4 + H * 4
    kv_per_pos = L * 2 * KVD * (2 if kv_f16 else 4)
    return weights, kv_per_pos


GATE_UP_BYTES = 2 * 11008 * 2048 // 2 + 2 * 11008 * 16 * 4 + 2048 * 4 + 11008 * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled DURING the timed region (read-only
    NVML queries from a thread every 2 ms, so a 20 ms region still holds ~10
    samples); nvidia-smi -lms 20 where NVML cannot be loaded."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, period_s=0.002):
        self.idx, self.period = gpu_index, period_s
        self.sms, self.mx, self.reasons = [], None, set()
        self.stop = None
        self.p = self.f = None

    def _poll(self, nv, h):
        bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                "sw_power_cap": 0x4}
        reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                self.sms.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                r = reasons_fn(h)
                for n, b in bits.items():
                    if r & b:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.idx)
            self.mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop = threading.Event()
            self.t = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.t.start()
        except Exception:
            self.stop = None
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self.p = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                           "--format=csv,noheader,nounits", "-lms", "20"],
                                          stdout=self.f, stderr=subprocess.DEVNULL)
            except Exception:
                self.p = None
        return self

    def __exit__(self, *a):
        if self.stop is not None:
            self.stop.set()
            self.t.join(timeout=2)
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        if self.f is not None:
            self.f.flush()
            self.f.seek(0)
            for line in self.f.read().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    self.sms.append(float(parts[1]))
                    self.mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(self.NAMES, parts[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(n)
            os.unlink(self.f.name)
            self.f = None
        return {"sm_mhz": statistics.median(self.sms) if self.sms else None, "sm_max_mhz": self.mx,
                "reasons": sorted(self.reasons), "samples": len(self.sms),
                "source": "nvml 2 ms" if self.stop is not None else "nvidia-smi 20 ms"}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return ws, rank, local


def max_over_ranks(ms, ws, device):
    """The job's time is the slowest rank's device time (weak scaling: every
    rank decodes its own sequences on its own replica)."""
    if ws <= 1:
        return ms
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    return float(t.item())


def job_throughput(ws, steps, ms):
    """Whole-job tok/s: every rank decoded `steps` tokens within `ms`."""
    return ws * steps / (ms / 1000.0)


def positions(start, period, n, cap):
    """Chunked start positions cycling in [start, start+period)."""
    out, done, pos = [], 0, start
    while done < n:
        k = min(cap, n - done, start + period - pos)
        out.append((pos, k))
        done += k
        pos += k
        if pos >= start + period:
            pos = start
    return out


def _decode_timed(rt, st, start, period, steps, warmup, cap):
    """warmup untimed + `steps` timed greedy tokens at positions cycling in
    [start, start + period) (decodeBatchAsync chains, ids stay on the
    device); returns the CUDA-event milliseconds on the runtime's stream."""
    import torch

    def decode(n):
        for pos, k in positions(start, period, n, cap):
            rt.decodeBatchAsync(pos, k)

    decode(warmup)
    rt.sync()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    decode(steps)
    e1.record(st)
    rt.sync()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def long_context(rt, st, cfg, ctx, steps, hbm):
    """f16 KV prefilled from a uniform-id prompt of `ctx` tokens,
    then `steps` greedy tokens at ctx..ctx+steps-1."""
    from vibethinker_webgpu_lora_b200.quantize import synth_ids
    prompt = synth_ids(ctx, PROMPT_SEED, cfg["vocabSize"])
    rt.prefillBatch(prompt)
    rt.argmaxLogits()
    ms = _decode_timed(rt, st, ctx, steps, steps, 3, 32)
    prof = [rt.profToken(int(prompt[-1]), ctx + 1) for _ in range(3)]
    attn_us = statistics.median(p["attn"] for p in prof) / cfg["numLayers"]
    weights, kv_per_pos = cfg_bytes(cfg)
    step_bytes = weights + kv_per_pos * (ctx + steps / 2)
    tok_s = steps / (ms / 1000.0)
    kv_layer = kv_per_pos // cfg["numLayers"] * (ctx + 1)
    return {"ctx": f"{ctx}..{ctx + steps}", "steps": steps, "value": round(tok_s, 2), "unit": "tok/s",
            "ms_per_step": round(ms / steps, 5),
            "step_roofline": {"bytes_per_step": int(step_bytes),
                              "frac": round(step_bytes * tok_s / 1e9 / hbm, 4),
                              "roofline_tok_s": round(hbm * 1e9 / step_bytes, 1)},
            "attention": {"us_per_layer": round(attn_us, 3), "kv_bytes_per_layer": int(kv_layer),
                          "achieved_gbs": round(kv_layer / (attn_us * 1e-6) / 1e9, 1),
                          "note": "profToken: eager launches, an event between categories"}}


def gemv_2048(hbm):
    """one int4 GEMV y = W x, W 2048 x 2048 ~ N(0, 0.02) quantised
    by the reference quantiser, x ~ N(0, 1), weights converted to the device
    layout once (as the model upload does).  72 launches captured in one CUDA
    graph with programmatic dependent launch: "cold" rotates over 72 distinct
    weight copies (161 MB > the 126 MB L2), "hot" reuses one copy."""
    import numpy as np
    import torch

    from vibethinker_webgpu_lora_b200 import kernels as K
    from vibethinker_webgpu_lora_b200.quantize import quantizeInt4Group, synth_normal
    N = Kd = 2048
    copies = 72
    W = synth_normal(N * Kd, 0xE6B00001, 0.02).reshape(N, Kd)
    x = torch.from_numpy(synth_normal(Kd, 0xE6B00002, 1.0)).cuda()
    p, s, _ = quantizeInt4Group(W)
    nb = K.q4_stream_bytes(N, Kd)
    nb_al = (nb + 255) // 256 * 256
    pool = torch.zeros(copies * nb_al, dtype=torch.uint8, device="cuda")
    tp, ts = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    for c in range(copies):
        K.q4_to_stream(tp, ts, N, Kd, pool[c * nb_al:])
    y = torch.zeros(N, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    out = {}
    for mode in ("cold", "hot"):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            for c in range(copies):  # warm the launch path outside the capture
                K.gemv_q4_stream(x, pool[(c if mode == "cold" else 0) * nb_al:], N, Kd, y, err, pdl=True)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for c in range(copies):
                K.gemv_q4_stream(x, pool[(c if mode == "cold" else 0) * nb_al:], N, Kd, y, err, pdl=True)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (reps * copies)
        out[mode] = {"us_per_gemv": round(us, 3), "achieved_gbs": round(2244608 / (us * 1e-6) / 1e9, 1),
                     "frac": round(2244608 / (us * 1e-6) / 1e9 / hbm, 4)}
    assert int(err.item()) == 0
    out.update({"bytes_per_gemv": 2244608, "launches": f"{copies} per graph, PDL chained",
                "note": "2 MiB nibbles + 128 KiB f32 scales + 8 KiB x + 8 KiB y per call"})
    return out


def run_ours(args, ws, rank, local):
    import torch

    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids

    cfg = E.QWEN25_3B
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        os.environ.setdefault("OMP_NUM_THREADS", str(max(1, (os.cpu_count() or 8) // ws)))
    long = args.ctx >= 1024
    # ctx ~128: prefill 96 ids, timed tokens cycle over 96..159
    n_prompt = args.ctx if long else 96
    period = 64
    extras = ws == 1 and not long and not args.no_extras
    max_ctx = max(n_prompt + period, 7800 + period if extras else 0) + 8
    cap = 32
    opts = {"maxCtx": max_ctx, "useF16": True, "device": local, "decodeBatchSize": cap}
    if args.path != "auto":
        opts["useFused"] = args.path == "fused"
    rt = E.QwenB200(cfg, opts).build("synthetic", seed=SEED)
    prompt = synth_ids(n_prompt, PROMPT_SEED ^ rank, cfg["vocabSize"])
    rt.prefillBatch(prompt)
    rt.argmaxLogits()
    st = torch.cuda.ExternalStream(rt.stream, device=dev)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    with Clocks(local) as ck:
        ms = _decode_timed(rt, st, n_prompt, period, args.steps, args.warmup, cap)
    ms = max_over_ranks(ms, ws, dev)
    clocks = ck.summary()
    launches = rt.lastDispatchCount * args.steps

    # dominant kernel (gate_up + SiLU GEMV) timed per launch with CUDA events
    # inside real decode steps (profToken brackets each kernel category)
    prof = [rt.profToken(int(prompt[-1]), n_prompt + 1) for _ in range(5)]
    gu_us = statistics.median(p["gate_up"] for p in prof) / cfg["numLayers"]
    step_us = statistics.median(sum(p.values()) for p in prof)

    # end to end through the public API with host buffers, configs[1] as
    # stated: prefillBatch(32 host ids) + argmaxLogits + 128 greedy tokens,
    # ids read back to the host after every decodeBatch call
    e2e_tokens = 128
    p32 = synth_ids(N_PROMPT, PROMPT_SEED ^ rank, cfg["vocabSize"])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rt.prefillBatch(p32)
    rt.argmaxLogits()
    done, pos = 0, N_PROMPT
    while done < e2e_tokens:
        got = rt.decodeBatch(pos, min(cap, e2e_tokens - done))
        done += len(got)
        pos += len(got)
    e2e_s = time.perf_counter() - t0

    weights, kv_per_pos = cfg_bytes(cfg)
    mean_ctx = n_prompt + period / 2
    step_bytes = weights + kv_per_pos * mean_ctx
    hbm, peak_kind = peaks()
    value = job_throughput(ws, args.steps, ms)
    ms_per_step = ms / args.steps
    achieved = GATE_UP_BYTES / (gu_us * 1e-6) / 1e9
    result = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4xf32",
        "data": "synthetic",
        "config": {"workload": f"configs[{2 if long else 1}]: Qwen2.5-3B-shape int4 greedy decode, "
                               f"batch 1, prefill {n_prompt} ids, timed tokens at ctx "
                               f"{n_prompt}..{n_prompt + period} (cycling)",
                   "kv": "f16", "scales": "f32 (stream layout: 16x128 blocks, interleaved f32 scales)", "lm_head": "int8 rows",
                   "l2": "inputs larger than L2 (1.79 GB of weights streamed per step)",
                   "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU"},
        "roofline": {"bound": "hbm", "kernel": "gate_up+SiLU int4 GEMV (22016x2048)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                     "bytes_per_launch": GATE_UP_BYTES, "launch_us": round(gu_us, 3),
                     # dram__bytes_read + dram__bytes_write of one gate_up launch, ncu
                     # --set full of `python bench.py --ncu-probe 4` (same kernel and shape)
                     "traffic": 24009984, "traffic_source": "ncu, bench.py --ncu-probe 4"},
        "step_roofline": {"bytes_per_step": int(step_bytes),
                          "achieved_gbs": round(step_bytes * value / ws / 1e9, 1),
                          "frac": round(step_bytes * value / ws / 1e9 / hbm, 4),
                          "roofline_tok_s": round(hbm * 1e9 / step_bytes, 1),
                          "profiled_step_us": round(step_us, 1),
                          "profiled_us_by_kernel": {k: round(statistics.median(p[k] for p in prof), 1)
                                                    for k in prof[0]}},
        "e2e": {"value": round(e2e_tokens / e2e_s, 2), "unit": "tok/s",
                "h2d_bytes_per_step": round(4 * N_PROMPT / e2e_tokens, 3),
                "d2h_bytes_per_step": 4,
                "what": f"prefillBatch({N_PROMPT} host ids) + argmaxLogits + decodeBatch to host, "
                        f"{e2e_tokens} tokens (ctx {N_PROMPT}..{N_PROMPT + e2e_tokens}), wall clock"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if extras:
        result["ctx4096"] = long_context(rt, st, cfg, 4096, 64, hbm)
        result["ctx7800"] = long_context(rt, st, cfg, 7800, 64, hbm)
        result["gemv_2048"] = gemv_2048(hbm)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg, n_prompt, args.cpu_steps)
    return result


BATCH_METRIC = "batched LoRA decode tok/s summed over 16 sequences (configs[4])"


def shard_sequences(total: int, rank: int, ws: int) -> list[int]:
    """The sequences rank `rank` of `ws` decodes: contiguous, every sequence
    on exactly one rank, sizes differing by at most one."""
    return list(range(total * rank // ws, total * (rank + 1) // ws))


def run_batch16(args, ws, rank, local):
    """16 sequences, each prefilled to 512 ids, then 64 sampled
    steps (top-k 40, T 0.7) with a rank-8 adapter (alpha 16) on all 252
    projections, hot-swapped for a second adapter at step 32.  Under
    torchrun the 16 sequences shard over the ranks (16 / N each, weights
    replicated, no collective): strong scaling, value = 16 x 64 tokens /
    the slowest rank's time.  Timed through the public API (eg_batch_sample:
    r uniforms in, ids out) with CUDA events on the runtime's stream; the
    prefill (511 batched steps) is the warm-up."""
    import numpy as np
    import torch

    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids, synth_uniform

    cfg = E.QWEN25_3B
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    total, n_prompt, steps, k, temp = 16, 512, 64, 40, 0.7
    mine = shard_sequences(total, rank, ws)
    n = len(mine)
    rt = E.QwenB200(cfg, {"maxCtx": n_prompt + steps + 8, "useF16": True, "useTcBatch": args.tc_batch,
                          "device": local}).build("synthetic", seed=SEED)
    a1 = E.synthetic_adapter(rt, 0xA1, rank=8, alpha=16)
    a2 = E.synthetic_adapter(rt, 0xA2, rank=8, alpha=16)
    rt.setLora(a1)
    rt.seqInit(n, n_prompt + steps + 2)
    slots = list(range(n))
    for sl, g in zip(slots, mine):
        rt.seqSetPrompt(sl, synth_ids(n_prompt, 0xE6B00100 + g, cfg["vocabSize"]))
    r = np.array([[synth_uniform(1, 0xE6B00200 ^ g ^ t)[0] for g in mine] for t in range(steps)],
                 np.float32)
    st = torch.cuda.ExternalStream(rt.stream, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rt.batchDecode(slots, n_prompt - 1)  # prefill: warm-up, untimed
    prefill_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as ck:
        t0 = time.perf_counter()
        e0.record(st)
        out1 = rt.batchSample(slots, steps // 2, k, temp, r[: steps // 2])
        rt.setLora(a2)  # hot swap at step 32
        out2 = rt.batchSample(slots, steps - steps // 2, k, temp, r[steps // 2:])
        e1.record(st)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    ms = max_over_ranks(e0.elapsed_time(e1), ws, dev)
    wall = max_over_ranks(wall * 1000.0, ws, dev) / 1000.0
    launches = rt.lastDispatchCount * steps
    weights, kv_per_pos = cfg_bytes(cfg)
    lora_bytes = 1662976 * cfg["numLayers"]
    step_bytes = weights + n * kv_per_pos * (n_prompt + steps / 2) + lora_bytes
    hbm, peak_kind = peaks()
    value = total * steps / (ms / 1000.0)
    achieved = step_bytes * steps / (ms / 1000.0) / 1e9
    assert out1.shape == (steps // 2, n) and out2.shape == (steps - steps // 2, n)
    a1.destroy()
    a2.destroy()
    return {
        "metric": BATCH_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": ws,
        "steps": steps, "warmup": n_prompt - 1, "ms_per_step": round(ms / steps, 4),
        "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
        "dtype": "int4xf32", "data": "synthetic",
        "config": {"workload": "configs[4]: 16 sequences x (prefill 512 + 64 sampled steps), "
                               "rank-8 LoRA on 252 projections, hot swap at step 32, top-k 40, T 0.7",
                   "kv": "f16", "lm_head": "int8 rows",
                   "l2": "inputs larger than L2 (1.79 GB of weights streamed per step)",
                   "parallelism": f"{n} sequences per GPU x {ws} GPUs (replicated weights)"},
        "roofline": {"bound": "hbm", "kernel": "whole batched step per GPU (weights once + its "
                                               "KV caches + LoRA A/B)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                     "bytes_per_launch": int(step_bytes), "traffic": None},
        "prefill": {"steps": n_prompt - 1, "s": round(prefill_s, 3),
                    "tok_s": round(n * (n_prompt - 1) / prefill_s, 1)},
        "e2e": {"value": round(total * steps / wall, 2), "unit": "tok/s",
                "h2d_bytes_per_step": total * 4, "d2h_bytes_per_step": total * 4,
                "what": "batchSample x2 (r uniforms H2D, ids D2H) + setLora, wall clock, max over ranks"},
        "gpu_launches": launches,
        "clocks": ck.summary(),
    }


PREFILL_METRIC = "prefill ms per prompt (configs[3], T=1024 and 4096)"


def run_prefill(args, local):
    """prefill of a T-token prompt (uniform ids) through the
    public API (prefillBatch: host ids in, last logits on the device), timed
    with CUDA events on the runtime's stream; T = 1024 and 4096, `--steps`
    prompts each after `--warmup` untimed ones.  One whole-prompt pass
    (the reference's _prefillFull): tcgen05 kind::f16 GEMMs for every
    projection and the tensor-core causal attention."""
    import torch

    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids

    cfg = E.QWEN25_3B
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    rt = E.QwenB200(cfg, {"maxCtx": 4096 + 64, "maxPrefillT": 4096, "useF16": True, "device": local}).build(
        "synthetic", seed=SEED)
    st = torch.cuda.ExternalStream(rt.stream, device=dev)
    steps = max(1, min(args.steps, 8))
    res = {}
    with Clocks(local) as ck:
        for T in (1024, 4096):
            p = synth_ids(T, PROMPT_SEED, cfg["vocabSize"])
            for _ in range(min(args.warmup, 3)):
                rt.prefillBatch(p)
            rt.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(steps):
                rt.prefillBatch(p)
            e1.record(st)
            rt.sync()
            torch.cuda.synchronize()
            res[T] = e0.elapsed_time(e1) / steps
    # tensor work of one T-row pass: the int4 projections' MACs, issued twice
    # (f16 hi and lo halves of the activations), plus the causal attention
    H, I, L = cfg["hiddenSize"], cfg["intermediateSize"], cfg["numLayers"]
    hd, nh, nkv = cfg["headDim"], cfg["numHeads"], cfg["numKVHeads"]
    params = L * ((nh + 2 * nkv) * hd * H + H * nh * hd + 2 * I * H + H * I)
    T = 4096
    gemm_flop = 2 * params * T * 2
    attn_flop = L * 4 * hd * nh * T * (T + 1) / 2
    tflops = (gemm_flop + attn_flop) / (res[T] / 1000.0) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, peak_kind = float(json.load(f)["bf16_tflops_sustained"]), "measured (bf16 cuBLAS, sustained)"
    except Exception:
        peak, peak_kind = 1400.0, "fallback"
    return {
        "metric": PREFILL_METRIC, "value": round(res[4096], 2), "unit": "ms",
        "per_T_ms": {str(T): round(v, 2) for T, v in res.items()},
        "tok_s": {str(T): round(T / (v / 1000.0), 1) for T, v in res.items()},
        "n_gpus": 1, "steps": steps, "warmup": min(args.warmup, 3),
        "ms_per_step": round(res[4096], 2), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4 x f16 hi/lo (f32 accumulate)", "data": "synthetic",
        "config": {"workload": "configs[3]: Qwen2.5-3B-shape prefill of a uniform-id prompt, "
                               "T = 1024 and 4096 (value: T = 4096), one whole-prompt pass", "kv": "f16",
                   "l2": "inputs larger than L2 (5.5 GB of f16 weight images per pass)",
                   "parallelism": "single GPU"},
        "roofline": {"bound": "tensor", "kernel": "whole prefill: tcgen05 kind::f16 GEMMs (hi + lo MMA "
                     "halves counted) + mma.sync attention", "achieved": round(tflops, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tflops / peak, 4), "peak_kind": peak_kind,
                     "traffic": None},
        "e2e": {"value": round(res[4096], 2), "unit": "ms", "h2d_bytes_per_step": 4 * 4096,
                "d2h_bytes_per_step": 0, "what": "prefillBatch from host ids"},
        "gpu_launches": 1 + 36 * 10 + 2,  # embed, 10 per layer, LM head, state
        "clocks": ck.summary(),
    }


def _oracle_decode(cfg, n_prompt, warmup, steps):
    """The reference's decode path restated in C (oracle/, f32 mimic of the
    WGSL kernels, OpenMP over rows on all host cores): prefill n_prompt
    uniform ids one position at a time (untimed), `warmup` untimed greedy
    tokens, then `steps` timed greedy tokens -- the same positions as the GPU
    arm's timed tokens.  Returns (tok/s, seconds, ctx range, cores)."""
    from oracle import oracle as O
    m = O.OracleModel(cfg, n_prompt + warmup + steps + 8, True, SEED)
    prompt = O.token_ids(n_prompt, PROMPT_SEED, cfg["vocabSize"])
    logits = None
    for t, tok in enumerate(prompt):
        logits = m.step(int(tok), t)
    tok, pos = O.argmax(logits), n_prompt
    for _ in range(warmup):
        tok = O.argmax(m.step(tok, pos))
        pos += 1
    p0 = pos
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = O.argmax(m.step(tok, pos))
        pos += 1
    s = time.perf_counter() - t0
    m.close()
    return steps / s, s, f"{p0}..{pos}", O.threads()


def cpu_baseline(cfg, n_prompt, steps):
    v, _, ctx, cores = _oracle_decode(cfg, n_prompt, 0, steps)
    return {"value": round(v, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{steps} greedy decode tokens of the full model at ctx {ctx} after an "
                      f"untimed {n_prompt}-token prefill (f32 mimic of the reference kernels, "
                      f"OpenMP over rows)"}


def run_reference(args, ws, rank):
    cfg = __import__("vibethinker_webgpu_lora_b200").QWEN25_3B
    n_prompt = args.ctx if args.ctx >= 1024 else 96
    steps = max(1, min(args.steps, args.cpu_steps))
    warm = min(args.warmup, 2)
    v, s, ctx, cores = _oracle_decode(cfg, n_prompt, warm, steps)
    sample = (f"{steps} greedy decode tokens of the full model at ctx {ctx} (prefill {n_prompt} "
              f"+ {warm} warm-up tokens untimed), the GPU arm's context")
    return {"metric": METRIC, "value": round(v, 3), "unit": "tok/s", "impl": "reference", "n_gpus": ws,
            "steps": steps, "warmup": warm, "ms_per_step": round(1000 * s / steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xf32",
            "data": "synthetic",
            "config": {"workload": f"configs[{2 if args.ctx >= 1024 else 1}] on the host CPU: "
                                   f"batch-1 greedy decode at ctx {ctx}"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def ncu_probe(ctx):
    """Smallest run that contains full decode steps, for ncu launch lists and
    single-kernel captures (the weights are 1.8 GB; nothing else is held)."""
    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids
    rt = E.QwenB200(E.QWEN25_3B, {"maxCtx": ctx + 40}).build("synthetic", seed=SEED)
    rt.prefillBatch(synth_ids(ctx, PROMPT_SEED, E.QWEN25_3B["vocabSize"]))
    rt.argmaxLogits()
    rt.decodeBatchAsync(ctx, 2)
    rt.sync()
    print(json.dumps({"ncu_probe": ctx, "launches_per_step": rt.lastDispatchCount}))


def ncu_probe_prefill(T):
    """Profiling target of the whole-prompt prefill: two prefillBatch calls
    of a T-token prompt (the first allocates the prefill scratch), exit."""
    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids
    cfg = E.QWEN25_3B
    rt = E.QwenB200(cfg, {"maxCtx": T + 8}).build("synthetic", seed=SEED)
    p = synth_ids(T, PROMPT_SEED, cfg["vocabSize"])
    rt.prefillBatch(p)
    rt.prefillBatch(p)
    rt.sync()
    print(json.dumps({"ncu_probe_prefill": T}))


def ncu_probe_gemm(T):
    """Profiling target of one whole-prompt tcgen05 GEMM launch shape: the
    down projection (2048 x 11008 int4, random words and scales) against T
    token rows, three calls, exit (a few tens of MB on the device)."""
    import numpy as np
    import torch

    from vibethinker_webgpu_lora_b200 import kernels as K
    N, Kd = 2048, 11008
    rng = np.random.default_rng(1)
    w = torch.from_numpy(rng.integers(0, 2 ** 32, N * Kd // 8, dtype=np.uint32)).cuda()
    sc = torch.from_numpy(rng.uniform(1e-3, 2e-3, N * (Kd // 128)).astype(np.float32)).cuda()
    ws = torch.zeros(K.q4_stream_bytes(N, Kd), dtype=torch.uint8, device="cuda")
    K.q4_to_stream(w, sc, N, Kd, ws)
    wc = torch.zeros(K.q4_tc_bytes(N, Kd), dtype=torch.uint8, device="cuda")
    K.q4_stream_to_tc(ws, N, Kd, wc)
    x = torch.randn(T, Kd, device="cuda")
    y = torch.empty(T, N, device="cuda")
    for _ in range(3):
        K.gemm_q4_stream(x, T, wc, N, Kd, y, use_tc=True)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_probe_gemm": T}))


def ncu_probe_attn(T):
    """Profiling target of the prefill attention: one KV layer of the 3B
    shape (16 query / 2 KV heads, f16 cache), a T-row pass from position 0,
    three calls, exit (tens of MB on the device)."""
    import torch

    from vibethinker_webgpu_lora_b200 import kernels as K
    nh, nkv, hd = 16, 2, 128
    g = torch.Generator(device="cuda").manual_seed(1)
    qkv0 = torch.randn(T, (nh + 2 * nkv) * hd, device="cuda", generator=g)
    kc = torch.zeros(T, nkv * hd, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    ang = torch.arange(T, device="cuda", dtype=torch.float32)[:, None] * torch.ones(hd, device="cuda")
    cos_t, sin_t = torch.cos(ang * 1e-3).contiguous(), torch.sin(ang * 1e-3).contiguous()
    out = torch.empty(T, nh * hd, device="cuda")
    for _ in range(3):
        qkv = qkv0.clone()
        K.attn_prefill(qkv, T, kc, vc, cos_t, sin_t, nh, nkv, 0, T, 1, out)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_probe_attn": T}))


def ncu_probe_batch(steps, tc=False):
    """Profiling target of the batched path as configs[4] runs it: a rank-8
    adapter on every projection, 16 slots with 8-token prompts, `steps`
    batched greedy steps (launches_per_step launches each), exit.  tc: the
    int4 GEMVs on the tcgen05 path."""
    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200.quantize import synth_ids
    cfg = E.QWEN25_3B
    rt = E.QwenB200(cfg, {"maxCtx": 128, "useTcBatch": tc}).build("synthetic", seed=SEED)
    rt.setLora(E.synthetic_adapter(rt, 0xA1, rank=8, alpha=16))
    rt.seqInit(16, 64)
    for sl in range(16):
        rt.seqSetPrompt(sl, synth_ids(8, 0xE6B00100 + sl, cfg["vocabSize"]))
    rt.batchDecode(list(range(16)), steps)
    print(json.dumps({"ncu_probe_batch": steps, "launches_per_step": rt.lastDispatchCount}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=128, choices=[128, 4096, 7800])
    ap.add_argument("--cpu-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the ctx 4096/7800 and configs[0] GEMV sub-objects")
    ap.add_argument("--path", default="auto", choices=["auto", "fused", "graph"],
                    help="decode path: persistent fused kernel or per-op CUDA graph")
    ap.add_argument("--workload", default="decode", choices=["decode", "batch16", "prefill", "gemm4", "attn"],
                    help="decode: configs[1]/[2] (the headline); batch16: configs[4]; "
                         "prefill: configs[3]")
    ap.add_argument("--tc-batch", action="store_true",
                    help="batch16: the batched int4 GEMVs on the tcgen05 path (useTcBatch)")
    ap.add_argument("--ncu-probe", type=int, default=0, metavar="CTX",
                    help="profiling target: build, prefill CTX tokens, decode 2 tokens, exit "
                         "(CTX * launches/step launches precede the 2 profiled steps)")
    args = ap.parse_args()
    if args.ncu_probe:
        if args.workload == "batch16":
            ncu_probe_batch(args.ncu_probe, args.tc_batch)
        elif args.workload == "prefill":
            ncu_probe_prefill(args.ncu_probe)
        elif args.workload == "gemm4":
            ncu_probe_gemm(args.ncu_probe)
        elif args.workload == "attn":
            ncu_probe_attn(args.ncu_probe)
        else:
            ncu_probe(args.ncu_probe)
        return
    if args.workload in ("gemm4", "attn"):
        ap.error(f"--workload {args.workload} is a profiling target: give --ncu-probe T")
    assert args.warmup >= 3, "at least 3 warm-up steps"
    ws, rank, local = dist_setup() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args, ws, rank)), flush=True)
        return
    if args.workload == "batch16":
        res = run_batch16(args, ws, rank, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.workload == "prefill":
        if rank == 0:
            print(json.dumps(run_prefill(args, local)), flush=True)
        return
    res = run_ours(args, ws, rank, local)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
