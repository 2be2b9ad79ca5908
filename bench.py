"""Q4-KV decode-attention benchmark (one JSON line on rank 0).

Default workload: multi-agent block-pool decode at scale, Llama-3.1-8B KV geometry, all
32 layers: 256 agents with context lengths drawn uniformly from [1024, 32768] (seeded),
K/V drawn N(0,1) in fp16 and quantized to group-64 Q4 into 256-token blocks scattered at
random pool offsets through per-agent block tables, one fp16 query token per agent.
A step = for every layer: quantize-on-append of the step's new K/V token of every agent,
then split-KV decode attention of every agent over its blocks.  Agents are partitioned
across ranks by balanced token count (greedy LPT); there is no collective on the data
path.  Weak scaling by default: a job on N GPUs is N x 256 agents drawn from the same
distribution and LPT-partitioned, so each rank decodes ~256 agents (the configuration's
per-GPU size); `--scaling strong` keeps the 256 agents fixed and gives each rank its share.

Other workloads (--workload): llama_layer, gemma, mla (single-instance decode), prefill
(Llama chunked prefill), gemma_prefill, mla_prefill (512-token chunks on the Gemma-3 and
MLA geometries) — the remaining shapes of the attention path, for their own measurement
lines; the default run also reports each of them under "configs".

`python bench.py --impl reference` times the CPU restatement of the same computation (the
reference's own MLX CPU path cannot run here: mlx is not installed) on a bounded sample.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LLAMA = dict(layers=32, hq=32, hkv=8, dk=128, dv=128)
GEMMA = dict(layers=48, hq=16, hkv=8, dk=256, dv=256, window=1024, global_every=6)
MLA = dict(layers=27, hq=16, hkv=16, dk=192, dv=128)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="multi_agent",
                   choices=["multi_agent", "llama_layer", "gemma", "mla", "prefill",
                            "gemma_prefill", "mla_prefill"])
    p.add_argument("--agents", type=int, default=256,
                   help="agents per GPU (weak scaling) or in total (strong scaling)")
    p.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                   help="weak: N GPUs decode N x --agents agents; strong: --agents in total")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--min-len", type=int, default=1024)
    p.add_argument("--max-len", type=int, default=32768)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--no-configs", action="store_true",
                   help="skip the per-configuration records after the headline")
    p.add_argument("--config-steps", type=int, default=5)
    return p.parse_args()


# ------------------------------------------------------------------------------- helpers


# DRAM bytes (read + write) per algorithmic byte of one decode launch, from the ncu capture
# of the 32-agent x 2-layer case of this workload (traffic grows with the Q4 bytes read).
DECODE_TRAFFIC_RATIO = 662.3 / 655.0


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1647.3)), \
            float(d.get("bf16_tflops_sustained", 1386.7)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed region.

    Read-only NVML queries from a background thread every 5 ms, plus one sample when the
    sampler starts and one when it stops, so short timed regions are covered; falls back to
    `nvidia-smi -lms 200` when NVML is unavailable.  Nothing here changes a GPU setting."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.samples: list[tuple[float, float, int]] = []
        self._nv = None
        self._handle = None
        self._stop = threading.Event()
        self._thread = None

    def _nvml_handle(self):
        import pynvml as nv

        nv.nvmlInit()
        try:
            import torch

            bus = torch.cuda.get_device_properties(self.index).pci_bus_id
            pci = f"{torch.cuda.get_device_properties(self.index).pci_domain_id:08x}:{bus:02x}:" \
                  f"{torch.cuda.get_device_properties(self.index).pci_device_id:02x}.0"
            h = nv.nvmlDeviceGetHandleByPciBusId(pci)
        except Exception:  # noqa: BLE001 - fall back to the NVML index
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
        return nv, h

    def _sample(self):
        nv, h = self._nv, self._handle
        try:
            self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                 float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                                 int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
        except Exception:  # noqa: BLE001
            pass

    def _loop(self):
        while not self._stop.wait(0.005):
            self._sample()

    def start(self):
        try:
            self._nv, self._handle = self._nvml_handle()
            self._sample()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
            return
        except Exception:  # noqa: BLE001 - no NVML: use nvidia-smi
            self._nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self._nv is not None:
            self._sample()
            self._stop.set()
            if self._thread is not None:
                self._thread.join(timeout=1)
            nv = self._nv
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            if not self.samples:
                return None
            reasons = sorted({k for _, _, r in self.samples for k, bit in bits.items() if r & bit})
            return {"sm_mhz": float(np.median([s for s, _, _ in self.samples])),
                    "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml"}
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxs.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sms:
            return None
        return {"sm_mhz": float(np.median(sms)), "sm_max_mhz": max(maxs),
                "reasons": sorted(reasons), "samples": len(sms), "source": "nvidia-smi"}


def agent_lengths(n_agents, lo, hi, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n_agents).tolist()


def job_agents(args, world):
    """Agents in the whole job: --agents per GPU under weak scaling, in total under strong."""
    return args.agents * world if args.scaling == "weak" else args.agents


def q4_bytes_per_token(hkv, dk, dv):
    return hkv * (dk // 2 + dk // 16 + dv // 2 + dv // 16)


# ------------------------------------------------------------------------------- our arm


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    am = load_package()
    am._lib.load()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.workload != "multi_agent":
        return run_single_workload(args, am, dev, rank, world)

    geo = LLAMA
    layers = args.layers or geo["layers"]
    hq, hkv, dk, dv = geo["hq"], geo["hkv"], geo["dk"], geo["dv"]
    n_total = job_agents(args, world)
    lengths_all = agent_lengths(n_total, args.min_len, args.max_len, args.seed)
    parts = am.lpt_partition(lengths_all, world)
    mine = sorted(parts[rank])
    lens = [lengths_all[i] for i in mine]
    A = len(mine)
    bt = 256
    # one extra token per agent: the step's appended token at position len
    blocks_per_layer = sum(-(-(n + 1) // bt) for n in lens)
    spec = am.ModelCacheSpec(n_layers=layers, n_kv_heads=hkv, head_dim=dk, block_tokens=bt,
                             layer_types=["global"] * layers)
    total_blocks = blocks_per_layer * layers
    alloc = am.shuffled_allocator(spec, total_blocks, seed=args.seed + 1 + rank)
    pool = am.PagedQ4Pool.for_spec(spec, total_blocks, torch.float16, dev)
    max_tokens = max(lens) + 1
    caches = [am.PagedLayerCache(pool, alloc, l, [f"agent{i}" for i in mine], max_tokens)
              for l in range(layers)]
    # fill: K/V ~ N(0,1) fp16, quantized into the blocks by the append kernel
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    t_fill = time.time()
    for l, c in enumerate(caches):
        for r, n in enumerate(lens):
            c.reserve(r, n + 1)
        for r, n in enumerate(lens):
            k = torch.randn(1, hkv, n, dk, generator=gen, device=dev, dtype=torch.float16)
            v = torch.randn(1, hkv, n, dv, generator=gen, device=dev, dtype=torch.float16)
            am.kernels.append(am.kernels.paged_view(pool.k, pool.v, c.table[r:r + 1]), k, v,
                              torch.zeros(1, dtype=torch.int32, device=dev))
        c.set_lengths([n + 1 for n in lens])
    torch.cuda.synchronize(dev)
    t_fill = time.time() - t_fill

    views = [c.view() for c in caches]
    pos = torch.tensor(lens, dtype=torch.int32, device=dev)       # new token position
    kv_len = torch.tensor([n + 1 for n in lens], dtype=torch.int32, device=dev)
    max_len = max(lens) + 1
    scale = dk ** -0.5
    q = torch.randn(layers, A, hq, 1, dk, generator=gen, device=dev, dtype=torch.float16)
    kn = torch.randn(layers, A, hkv, 1, dk, generator=gen, device=dev, dtype=torch.float16)
    vn = torch.randn(layers, A, hkv, 1, dv, generator=gen, device=dev, dtype=torch.float16)
    out = torch.empty(layers, A, hq, 1, dv, device=dev, dtype=torch.float16)
    stream = torch.cuda.current_stream(dev)

    # Per-call CUDA events on a sample of the layers only: an event recorded between two
    # kernels keeps the second from launching before the first ends (programmatic stream
    # serialization overlaps consecutive kernels), so events around every call would slow
    # the timed step itself; every layer's calls have the same shapes.
    ev_layers = list(range(0, layers, 8))

    def step(ev=None):
        for l in range(layers):
            timed = ev is not None and l in ev
            if timed:
                ev[l][2].record(stream)
            am.kernels.append(views[l], kn[l], vn[l], pos)
            if timed:
                ev[l][0].record(stream)
            am.kernels.attention(views[l], q[l], scale, kv_len, max_len, out=out[l],
                                 mode="decode")
            if timed:
                ev[l][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    evs = [{l: [torch.cuda.Event(enable_timing=True) for _ in range(3)] for l in ev_layers}
           for _ in range(args.steps)]
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.nvtx.range_push("timed")
    t0.record(stream)
    for s in range(args.steps):
        step(evs[s])
    t1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1)
    attn_ms = [evs[s][l][0].elapsed_time(evs[s][l][1]) for s in range(args.steps)
               for l in ev_layers]
    append_ms = [evs[s][l][2].elapsed_time(evs[s][l][0]) for s in range(args.steps)
                 for l in ev_layers]
    ms_max = ms_local
    if world > 1:
        tt = torch.tensor([ms_local], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt.item())
    ms_per_step = ms_max / args.steps
    tokens_per_step = n_total if world > 1 or A == n_total else A
    value = tokens_per_step / (ms_per_step / 1e3)

    # roofline of the decode attention call (split-KV kernel, plus the combine kernel when
    # split chunks are merged through the workspace instead of inside a cluster)
    combine = am.kernels.decode_workspace_bytes(views[0], A, hq, 1, max_len) > 0
    per_tok = q4_bytes_per_token(hkv, dk, dv)
    launch_bytes = sum(n + 1 for n in lens) * per_tok + A * hq * (dk + dv) * 2
    avg_launch_s = float(np.mean(attn_ms)) / 1e3
    hbm, _, _, peak_kind = peaks()
    achieved = launch_bytes / avg_launch_s / 1e9
    # quantize-on-append of the step's token: per agent and KV head, fp16 K and V rows read,
    # their Q4 codes, scales and biases written
    append_bytes = A * hkv * (2 * (dk + dv) + q4_bytes_per_token(1, dk, dv))
    append_s = float(np.mean(append_ms)) / 1e3
    append_roof = {"kernel": "am_q4_append (append_kernel), one token per agent", "bound": "hbm",
                   "achieved": round(append_bytes / append_s / 1e9, 1), "peak": hbm,
                   "peak_kind": peak_kind, "unit": "GB/s",
                   "frac": round(append_bytes / append_s / 1e9 / hbm, 4),
                   "bytes_per_launch": int(append_bytes), "avg_launch_ms": round(append_s * 1e3, 5),
                   "note": "one launch moves %.2f MB: latency-bound; see the prefill record for "
                           "a 512-token chunk" % (append_bytes / 1e6)}

    # e2e: host (pinned) queries and new K/V -> device, outputs -> host, every step
    e2e = None
    if not args.no_e2e:
        hq_buf = q.cpu().pin_memory()
        hk_buf = kn.cpu().pin_memory()
        hv_buf = vn.cpu().pin_memory()
        ho_buf = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        dq, dk_, dv_ = torch.empty_like(q), torch.empty_like(kn), torch.empty_like(vn)

        # Copies run on their own stream, pipelined with the layers as a serving loop would:
        # every layer's inputs go up at the start of the step (one event per layer, so layer
        # l starts as soon as its own inputs landed), and each layer's output goes down as
        # soon as that layer is done.  The step ends when its last output is on the host.
        copy_stream = torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(layers)]
        layer_done = [torch.cuda.Event() for _ in range(layers)]

        def e2e_step():
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_stream(stream)  # the previous step is done with the buffers
                for l in range(layers):
                    dq[l].copy_(hq_buf[l], non_blocking=True)
                    dk_[l].copy_(hk_buf[l], non_blocking=True)
                    dv_[l].copy_(hv_buf[l], non_blocking=True)
                    in_ready[l].record(copy_stream)
            for l in range(layers):
                stream.wait_event(in_ready[l])
                am.kernels.append(views[l], dk_[l], dv_[l], pos)
                am.kernels.attention(views[l], dq[l], scale, kv_len, max_len, out=out[l],
                                     mode="decode")
                layer_done[l].record(stream)
            with torch.cuda.stream(copy_stream):
                for l in range(layers):
                    copy_stream.wait_event(layer_done[l])
                    ho_buf[l].copy_(out[l], non_blocking=True)
            stream.wait_stream(copy_stream)

        for _ in range(max(args.warmup, 3)):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        h2d = (q.numel() + kn.numel() + vn.numel()) * 2
        d2h = out.numel() * 2
        e2e = {"value": round(tokens_per_step / (e_ms / args.steps / 1e3), 2), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "path": "PagedLayerCache views via the C ABI (am_q4_append + am_q4_decode); "
                       "per-layer host copies on a second stream, pipelined with the layers"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_multi_agent(args, lengths_all, layers, geo, budget_s=args.cpu_seconds)

    # The other configurations, each timed briefly in this process after the headline (one
    # GPU: they are single-instance shapes, replicas across GPUs).  The 256-agent pool is
    # released first: together they would not fit in HBM.
    pool_gb = pool.nbytes / 1e9
    sub = None
    if world == 1 and not args.no_configs:
        del caches, views, pool, alloc, q, kn, vn, out
        if not args.no_e2e:
            del hq_buf, hk_buf, hv_buf, ho_buf, dq, dk_, dv_
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
        sub = {}
        for w in ("llama_layer", "gemma", "mla", "prefill", "gemma_prefill", "mla_prefill"):
            # each record on its own: a configuration that fails (out of memory on a shared
            # box, say) is reported as such and does not take the headline line with it
            try:
                sub[w] = measure_config(w, am, dev, steps=args.config_steps, warmup=3, seed=args.seed)
            except Exception as e:  # noqa: BLE001 - reported in the line, never swallowed silently
                sub[w] = {"error": f"{type(e).__name__}: {e}"[:300]}
            try:
                torch.cuda.synchronize(dev)
                torch.cuda.empty_cache()
            except Exception as e:  # noqa: BLE001 - a broken context ends the remaining records
                sub["stopped"] = f"{type(e).__name__}: {e}"[:300]
                break

    if rank == 0:
        line = {
            "metric": "Q4-KV decode attention tokens/s (whole job) and achieved HBM GB/s vs peak",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: seeded N(0,1) fp16 K/V/queries, Q4 group-64 (no dataset)",
            "config": {"workload": "multi_agent_block_pool_decode", "model_shape": "Llama-3.1-8B KV",
                       "agents": n_total, "agents_this_rank0": A, "layers": layers,
                       "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": dk,
                       "context": f"U[{args.min_len},{args.max_len}] seed {args.seed}",
                       "total_context_tokens": int(sum(lengths_all)), "block_tokens": bt,
                       "blocks": "random pool offsets", "parallelism": f"agent-sharded x{world} (LPT)",
                       "step": "per layer: append 1 token/agent + split-KV decode",
                       "l2": "inputs larger than L2 (Q4 cache %.1f GB/rank)" % pool_gb,
                       "fill_s": round(t_fill, 1)},
            "roofline": {"kernel": "am_q4_decode (decode_kernel%s)" % (
                             " + combine_kernel" if combine else ", chunks merged in-cluster"),
                         "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "bytes_per_launch": int(launch_bytes),
                         "avg_launch_ms": round(avg_launch_s * 1e3, 4),
                         "launch_timing": "CUDA events around the calls of layers %s of every "
                                          "timed step (events between calls break the launch "
                                          "overlap, so not every layer carries them)" % ev_layers,
                         "traffic": round(launch_bytes * DECODE_TRAFFIC_RATIO),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                           "decode launch of the 32-agent case (662.3 MB for 655.0 MB "
                                           "algorithmic), scaled by the bytes this launch processes"},
            "e2e": e2e,
            "gpu_launches": args.steps * layers * (3 if combine else 2),
            "clocks": clk,
            "cpu_baseline": cpu,
            "append_roofline": append_roof,
            "configs": sub,
        }
        print(json.dumps(line))


def measure_config(w, am, dev, steps=5, warmup=3, seed=0, layers_override=None):
    """One of the single-instance configurations, timed on this GPU; returns its record.

    llama_layer / gemma / mla: decode attention over a contiguous Q4 cache (one Llama layer,
    the Gemma-3 step, the MLA step),
    the whole step (every layer or rotating instance) captured in one CUDA graph, so the
    time is device time; per-call time = step / calls.
    prefill / gemma_prefill / mla_prefill: per layer, a 512-token chunk's K/V quantized and
    appended into 256-token pool blocks at shuffled offsets (am_q4_append), then causal
    attention of the chunk over the cached prefix plus itself (am_q4_prefill: dequantize
    stage + tcgen05 attention); launched eagerly with CUDA events around every call.
    """
    import torch

    gen = torch.Generator(device=dev).manual_seed(seed)
    if w == "llama_layer":
        B, layers, N, L = 2, 1, 2048, 1
        hq, hkv, dk, dv, window = 32, 8, 128, 128, 0
        reps = 256  # rotating instances so the working set exceeds L2
    elif w == "gemma":
        B, layers, N, L = 8, GEMMA["layers"], 4096, 1
        hq, hkv, dk, dv, window = 16, 8, 256, 256, GEMMA["window"]
        reps = 1
    elif w == "mla":
        B, layers, N, L = 16, MLA["layers"], 8192, 1
        hq, hkv, dk, dv, window = 16, 16, 192, 128, 0
        reps = 1
    elif w in PREFILL_SHAPES:
        return measure_prefill(am, dev, steps, warmup, gen, w)
    else:
        raise ValueError(w)
    if layers_override and w != "llama_layer":
        layers = layers_override  # a shorter step of the same layer shapes (profiling)
    inst = layers * reps
    qdt = torch.float16
    kv = []
    for _ in range(inst):
        k = torch.randn(B, hkv, N, dk, generator=gen, device=dev, dtype=qdt)
        v = torch.randn(B, hkv, N, dv, generator=gen, device=dev, dtype=qdt)
        kv.append((am.quantize(k), am.quantize(v)))
        del k, v
    views = [am.kernels.contiguous_view(kq, vq)[0] for kq, vq in kv]
    q = torch.randn(inst, B, hq, L, dk, generator=gen, device=dev, dtype=qdt)
    out = torch.empty(inst, B, hq, L, dv, device=dev, dtype=qdt)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=dev)
    is_global = [(l % GEMMA["global_every"]) == GEMMA["global_every"] - 1 for l in range(layers)]
    stream = torch.cuda.current_stream(dev)

    def win(i):
        return 0 if (w != "gemma" or is_global[i % layers]) else window

    def step():
        for i in range(inst):
            am.kernels.attention(views[i], q[i], dk ** -0.5, kv_len, N, causal=True,
                                 window=win(i), out=out[i], mode="decode")

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    step_ms = t0.elapsed_time(t1) / steps
    ms = step_ms / reps
    launch_ms = step_ms / inst  # graph nodes run back to back: mean time per attention call
    # kernel launches per step: one per call, plus a combine launch for split decode calls
    # whose chunks merge through the workspace
    launches = sum(1 + (am.kernels.decode_workspace_bytes(views[i], B, hq, L, N, window=win(i)) > 0)
                   for i in range(inst))
    hbm, _, _, kind = peaks()
    per_tok = q4_bytes_per_token(hkv, dk, dv)
    keys = [N if win(l) == 0 else min(N, window) for l in range(layers)]
    step_bytes = sum(keys) * B * per_tok + layers * B * hq * (dk + dv) * 2
    achieved = step_bytes / layers / (launch_ms / 1e3) / 1e9
    del graph, views, kv, q, out
    torch.cuda.empty_cache()
    return {"metric": "decode tokens/s", "value": round(B / (ms / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(ms, 4), "steps": steps, "dtype": "f16",
            "config": {"workload": w, "batch": B, "layers": layers, "context": N,
                       "n_q_heads": hq, "n_kv_heads": hkv, "k_dim": dk, "v_dim": dv,
                       "window": window,
                       "l2": f"{reps} rotating instances" if reps > 1 else "inputs larger than L2",
                       "timing": "whole step in one CUDA graph; per-call time = step / calls"},
            "roofline": {"kernel": "am_q4_decode", "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": hbm, "peak_kind": kind, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "avg_launch_ms": round(launch_ms, 5),
                         "bytes_per_launch": int(step_bytes / layers)},
            "gpu_launches": steps * launches, "clocks": clk}


PREFILL_SHAPES = {
    # 512-token bf16 chunks over a cached Q4 prefix, one per model geometry
    "prefill": dict(model="Llama-3.1-8B", B=2, P=4096, window=0, global_every=1, **LLAMA),
    "gemma_prefill": dict(model="Gemma-3-12B", B=8, P=4096, **GEMMA),
    "mla_prefill": dict(model="DeepSeek-Coder-V2-Lite (MLA)", B=16, P=8192, window=0,
                        global_every=1, **MLA),
}


def measure_prefill(am, dev, steps, warmup, gen, workload="prefill"):
    """Chunked prefill of a 512-token bf16 chunk over a cached Q4 prefix (one geometry)."""
    import torch

    g = PREFILL_SHAPES[workload]
    B, layers, P, L = g["B"], g["layers"], g["P"], 512
    hq, hkv, dk, dv = g["hq"], g["hkv"], g["dk"], g["dv"]
    window, every = g["window"], g["global_every"]
    is_global = [window == 0 or (l % every) == every - 1 for l in range(layers)]
    N, bt = P + L, 256
    spec = am.ModelCacheSpec(n_layers=layers, n_kv_heads=hkv, head_dim=dk, block_tokens=bt,
                             layer_types=["global"] * layers)
    blocks = layers * B * (-(-N // bt))
    alloc = am.shuffled_allocator(spec, blocks, seed=7)
    pool = am.PagedQ4Pool(hkv, dk, dv, blocks, bt, torch.bfloat16, dev)
    caches = [am.PagedLayerCache(pool, alloc, l, [f"a{r}" for r in range(B)], N)
              for l in range(layers)]
    bf = torch.bfloat16
    for c in caches:
        c.append(torch.randn(B, hkv, P, dk, generator=gen, device=dev, dtype=bf),
                 torch.randn(B, hkv, P, dv, generator=gen, device=dev, dtype=bf))
        for r in range(B):
            c.reserve(r, N)
        c.set_lengths([N] * B)
    views = [c.view() for c in caches]
    kc = torch.randn(layers, B, hkv, L, dk, generator=gen, device=dev, dtype=bf)
    vc = torch.randn(layers, B, hkv, L, dv, generator=gen, device=dev, dtype=bf)
    q = torch.randn(layers, B, hq, L, dk, generator=gen, device=dev, dtype=bf)
    out = torch.empty(layers, B, hq, L, dv, device=dev, dtype=bf)
    pos = torch.full((B,), P, dtype=torch.int32, device=dev)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=dev)
    # The cached prefix of layer l + 1 is dequantized into the workspace on a side stream
    # while layer l runs (am_q4_prefill_stage over keys [0, P)); on the layer's own path
    # only the appended chunk is staged (keys [P, end)) before the attention kernel
    # (am_q4_prefill_attend).  Two workspaces alternate between layers.  The layers run on
    # a high-priority stream, so the side stream's stage blocks only take SMs the layer's
    # kernels leave free.
    lib = am._lib.load()
    lowest, highest = torch.cuda.Stream.priority_range()
    stream = torch.cuda.Stream(dev, priority=highest)
    side = torch.cuda.Stream(dev, priority=lowest)
    stream.wait_stream(torch.cuda.current_stream(dev))
    prev_stream = torch.cuda.current_stream(dev)
    torch.cuda.set_stream(stream)
    try:
        win = [0 if is_global[l] else window for l in range(layers)]
        args = [am.kernels.attention_args(views[l], q[l], dk ** -0.5, kv_len, N, causal=True,
                                          window=win[l], out=out[l]) for l in range(layers)]
        nbytes = max(am.kernels.prefill_workspace_bytes(views[l], B, hq, L, N, window=win[l])
                     for l in range(layers))
        ws = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
        pre_done = [torch.cuda.Event() for _ in range(layers)]
        chunk_done = [torch.cuda.Event() for _ in range(layers)]
        s_main, s_side = stream.cuda_stream, side.cuda_stream

        def stage(l, lo, hi, st):
            rc = lib.am_q4_prefill_stage(ctypes.byref(views[l].desc), ctypes.byref(args[l][0]), lo, hi,
                                         ws[l % 2].data_ptr(), nbytes, st)
            am._lib.check("am_q4_prefill_stage", rc)

        def step(ev=None):
            side.wait_stream(stream)  # the previous step's layers are done with both workspaces
            stage(0, 0, P, s_side)
            pre_done[0].record(side)
            for l in range(layers):
                if ev is not None:
                    ev[l][0].record(stream)
                am.kernels.append(views[l], kc[l], vc[l], pos)
                if ev is not None:
                    ev[l][1].record(stream)
                stream.wait_event(pre_done[l])
                stage(l, P, 2 ** 31 - 1, s_main)
                chunk_done[l].record(stream)
                rc = lib.am_q4_prefill_attend(ctypes.byref(views[l].desc), ctypes.byref(args[l][0]),
                                              ws[l % 2].data_ptr(), nbytes, s_main)
                am._lib.check("am_q4_prefill_attend", rc)
                if l + 1 < layers:
                    # from here on the layer's stream runs only the attention kernel, and
                    # workspace (l + 1) % 2 is free (layer l - 1's attention came before)
                    side.wait_event(chunk_done[l])
                    stage(l + 1, 0, P, s_side)
                    pre_done[l + 1].record(side)
                if ev is not None:
                    ev[l][2].record(stream)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(layers)]
               for _ in range(steps)]
        clocks = ClockSampler(dev.index)
        clocks.start()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for s in range(steps):
            step(evs[s])
        t1.record(stream)
        torch.cuda.synchronize(dev)
        clk = clocks.stop()
        ms = t0.elapsed_time(t1) / steps
        attn_ms = float(np.mean([evs[s][l][1].elapsed_time(evs[s][l][2]) for s in range(steps)
                                 for l in range(layers)]))
        app_ms = float(np.mean([evs[s][l][0].elapsed_time(evs[s][l][1]) for s in range(steps)
                                for l in range(layers)]))
    finally:
        torch.cuda.set_stream(prev_stream)
    hbm, _, tf_sus, kind = peaks()
    # visible (query, key) pairs per (sequence, head): causal over prefix + chunk, and for a
    # window layer only the last `window` positions up to each query
    def pairs(w):
        return sum(min(P + i + 1, w) if w else P + i + 1 for i in range(L))
    flops = sum(2 * B * hq * (dk + dv) * pairs(0 if is_global[l] else window)
                for l in range(layers)) / layers
    app_bytes = B * hkv * L * (2 * (dk + dv) + q4_bytes_per_token(1, dk, dv))
    del caches, views, pool, kc, vc, q, out
    torch.cuda.empty_cache()
    return {"metric": "prefill tokens/s", "value": round(B * L / (ms / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(ms, 4), "steps": steps, "dtype": "bf16",
            "config": {"workload": workload, "model_shape": g["model"], "batch": B,
                       "layers": layers, "prefix": P, "q_len": L, "n_q_heads": hq,
                       "n_kv_heads": hkv, "k_dim": dk, "v_dim": dv,
                       "window": window, "global_layers": sum(is_global),
                       "cache": "256-token paged blocks at shuffled offsets",
                       "step": "per layer: append the chunk (am_q4_append), dequantize its rows "
                               "(am_q4_prefill_stage) and attend (am_q4_prefill_attend); the cached "
                               "prefix of the next layer is dequantized on a side stream meanwhile",
                       "timing": "eager launches; CUDA events around every append and every "
                                 "stage + attention on the layer's stream"},
            "roofline": {"kernel": "am_q4_prefill_stage (chunk rows) + am_q4_prefill_attend (%s), "
                                   "prefix staged on a side stream" % (
                             "prefill2_kernel" if dk <= 128 and dv <= 128 else "prefill_kernel"),
                         "flops_per_launch_note": "layer mean of 2 * B * Hq * (Dk + Dv) * visible pairs",
                         "bound": "tensor", "achieved": round(flops / (attn_ms / 1e3) / 1e12, 2),
                         "peak": tf_sus, "peak_kind": kind + " sustained bf16", "unit": "TFLOP/s",
                         "frac": round(flops / (attn_ms / 1e3) / 1e12 / tf_sus, 4),
                         "flops_per_launch": int(flops), "avg_launch_ms": round(attn_ms, 5)},
            "append_roofline": {"kernel": "am_q4_append (append_kernel), 512-token chunk",
                                "bound": "hbm",
                                "achieved": round(app_bytes / (app_ms / 1e3) / 1e9, 1),
                                "peak": hbm, "peak_kind": kind, "unit": "GB/s",
                                "frac": round(app_bytes / (app_ms / 1e3) / 1e9 / hbm, 4),
                                "bytes_per_launch": int(app_bytes),
                                "avg_launch_ms": round(app_ms, 5)},
            "gpu_launches": steps * layers * 4, "clocks": clk}


def run_single_workload(args, am, dev, rank, world):
    """One single-instance workload on its own (replicas across ranks: every rank runs the
    same instance)."""
    import torch
    import torch.distributed as dist

    rec = measure_config(args.workload, am, dev, steps=args.steps, warmup=args.warmup, seed=args.seed,
                         layers_override=args.layers)
    ms = rec["ms_per_step"]
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    per_step = rec["value"] * rec["ms_per_step"] / 1e3  # tokens one instance produces per step
    if rank == 0:
        rec.update({"metric": f"Q4 attention {args.workload}: {rec['metric']}",
                    "value": round(per_step * world / (ms / 1e3), 2), "n_gpus": world,
                    "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "data": "synthetic: seeded N(0,1)"})
        rec["config"]["parallelism"] = f"replicas x{world}"
        print(json.dumps(rec))


# ------------------------------------------------------------------------------- CPU arm


def cpu_baseline_multi_agent(args, lengths_all, layers, geo, budget_s=12.0, threads=None,
                             sampler=None):
    """Time the C oracle (OpenMP over agents x KV heads, all host threads) on a bounded
    sample of the workload: one layer of decode for a sample of agents held in a paged Q4
    pool (256-token blocks, random block order), repeated until the time budget is spent;
    the rate is extrapolated by Q4 bytes to the full step (all agents, all layers).
    `sampler` (from cpu_sampler) reuses an already built sample."""
    run = sampler or cpu_sampler(lengths_all, layers, geo, threads)
    return run(budget_s)


def cpu_sampler(lengths_all, layers, geo, threads=None):
    """Build the CPU baseline's sample once; returns budget_s -> result dict."""
    from oracle import q4_oracle as orc

    orc.build()
    # all host threads this process may use (launchers such as torchrun default OpenMP to 1)
    orc.set_threads(threads or len(os.sched_getaffinity(0)))
    nthr = orc.num_threads()
    hq, hkv, dk, dv = geo["hq"], geo["hkv"], geo["dk"], geo["dv"]
    rng = np.random.default_rng(1234)
    per_tok = q4_bytes_per_token(hkv, dk, dv)
    bt = 256
    sample = [n + 1 for n in lengths_all[: max(1, min(len(lengths_all), (nthr + hkv - 1) // hkv * 2, 32))]]
    nblk = [-(-n // bt) for n in sample]
    total = sum(nblk)
    perm = rng.permutation(total).astype(np.int32)
    table = np.full((len(sample), max(nblk)), -1, np.int32)
    o = 0
    for i, nb in enumerate(nblk):
        table[i, :nb] = perm[o:o + nb]
        o += nb
    k = rng.standard_normal((total, hkv, bt, dk), dtype=np.float32).astype(np.float16)
    kq = orc.quantize(k.view(np.uint16))
    del k
    v = rng.standard_normal((total, hkv, bt, dv), dtype=np.float32).astype(np.float16)
    vq = orc.quantize(v.view(np.uint16))
    del v
    q = rng.standard_normal((len(sample), hq, 1, dk), dtype=np.float32)
    kv_len = np.array(sample, np.int32)

    sample_bytes = sum(sample) * per_tok
    full_bytes = sum(n + 1 for n in lengths_all) * per_tok * layers

    def once():
        """One decode pass of one layer over the sample; returns its wall time in seconds."""
        t = time.perf_counter()
        orc.attention(q, kq, vq, dk ** -0.5, n_kv_heads=hkv, layout=1, block_table=table,
                      kv_len=kv_len, causal=False)
        return time.perf_counter() - t

    def run(budget_s):
        done_s, reps = 0.0, 0
        while done_s < budget_s or reps == 0:
            done_s += once()
            reps += 1
        done_bytes = sample_bytes * reps
        step_s = done_s * full_bytes / done_bytes
        return {"value": round(len(lengths_all) / step_s, 3), "unit": "tokens/s",
                "cores": min(nthr, len(sample) * hkv), "kind": "port",
                "sample": f"{len(sample)} agents x 1 layer decode over a paged Q4 pool, {reps} reps "
                          f"({done_bytes / 1e9:.2f} GB of Q4 K/V in {done_s:.1f} s), extrapolated "
                          f"by Q4 bytes to {len(lengths_all)} agents x {layers} layers",
                "achieved_gbs": round(done_bytes / done_s / 1e9, 2)}

    run.once = once
    run.fraction = sample_bytes / full_bytes  # share of a full step's Q4 bytes in one pass
    run.sample_agents = len(sample)
    run.cores = min(nthr, len(sample) * hkv)
    return run


def run_reference(args, rank, world):
    """The reference arm: the C restatement of the path on the host cores (the reference's own
    CPU backend, mlx, is not installed).  A step is one decode pass of one layer over a sample
    of agents held in a paged Q4 pool, timed as it runs; its tokens/s counts the step as the
    share of the full job's Q4 bytes it reads (the job's agents x 32 layers x 144 B per token
    per KV head), so ms_per_step is the measured time of the sample step."""
    if rank != 0:
        return
    geo = LLAMA
    layers = args.layers or geo["layers"]
    lengths_all = agent_lengths(job_agents(args, world), args.min_len, args.max_len, args.seed)
    sampler = cpu_sampler(lengths_all, layers, geo)  # the sample is built once, then timed
    for _ in range(args.warmup):
        sampler.once()
    t0 = time.time()
    step_s = [sampler.once() for _ in range(args.steps)]
    wall = time.time() - t0
    ms = float(np.mean(step_s)) * 1e3
    tokens_per_step = len(lengths_all) * sampler.fraction
    value = tokens_per_step / (ms / 1e3)
    per_tok = q4_bytes_per_token(geo["hkv"], geo["dk"], geo["dv"])
    step_gb = sum(n + 1 for n in lengths_all) * per_tok * layers * sampler.fraction / 1e9
    print(json.dumps({
        "impl": "reference",
        "metric": "Q4-KV decode attention tokens/s (whole job) and achieved HBM GB/s vs peak",
        "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,1) fp16 K/V/queries, Q4 group-64",
        "config": {"workload": "multi_agent_block_pool_decode", "agents": len(lengths_all),
                   "layers": layers, "context": f"U[{args.min_len},{args.max_len}]",
                   "step": f"1 layer of decode over {sampler.sample_agents} agents' paged Q4 "
                           f"blocks ({step_gb:.3f} GB, {100 * sampler.fraction:.3f}% of a full "
                           f"step's Q4 bytes); tokens per step counted by that share"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": sampler.cores,
                         "kind": "port",
                         "sample": f"{sampler.sample_agents} agents x 1 layer per step, "
                                   f"{args.steps} timed steps"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "achieved_gbs": round(step_gb / (ms / 1e3), 2),
        "note": "mlx (the reference's CPU backend) is not installed; the C/OpenMP restatement "
                "of the path is timed on the host cores instead",
        "wall_s": round(wall, 2)}))


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
