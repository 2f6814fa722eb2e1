"""Benchmark of the non-GEMM Phi-tiny-MoE prefill path on B200.

Workload: 64 prompts x 2048 tokens (ids uniform over
the 32064-token vocabulary, seed 4), prefix-trie dedup, all 32 layers'
non-GEMM ops (embedding gather, LayerNorms, RoPE, attn += x + LayerNorm,
top-2 routing + permutation, SiLU(gate) * up, un-permute fused with the
carried add + LayerNorm), final add + LayerNorm, expansion to token rows and
-- on N > 1 GPUs -- one NCCL gather of the final hidden states
[64 x 2048, 4096] to rank 0. Prompts are sharded across ranks (strong
scaling: the 64-prompt batch is fixed). GEMM outputs are seeded N(0,1)
stand-ins of the config.h shapes, a pool of them reused round-robin across
the 32 layers (each set far larger than L2).

One "step" = that whole pass. `value` is tokens/s over all ranks with the
inputs resident in HBM; `e2e` is the same step through the public API from
host token ids (host trie build, H2D of the index arrays, D2H of the last-
token hidden states). `--impl reference` times the reference's own host
implementation of the path (oracle/_ref) on a bounded sample instead.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "non-GEMM prefill tokens/s (64x2048 prompts, 32 layers; layer-op HBM GB/s in roofline)"
# DRAM bytes (read + write) per node row of a kernel launch, from one ncu
# capture of that kernel on a smaller case of the same workload (32,768 rows),
# scaled to a launch by rows.
TRAFFIC_BYTES_PER_ROW = {"fused": (1611.028480e6 + 1017.303808e6) / 32768}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--exact", action="store_true", help="B2_FLAG_EXACT_ORDER reductions")
    p.add_argument("--prompts", type=int, default=64)
    p.add_argument("--length", type=int, default=2048)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--pool", type=int, default=0, help="stand-in sets (0 = fit to memory)")
    p.add_argument("--chunks", type=int, default=0, help="sub-batches per rank (0 = 1 on one GPU, 3 otherwise)")
    p.add_argument("--no-graph", action="store_true",
                   help="configs 1-4: launch the op chain eagerly instead of replaying a CUDA graph of it")
    p.add_argument("--serial-chunks", action="store_true",
                   help="run a rank's chunks one after another on one stream (default: concurrent streams, "
                        "chunk 0 at the highest priority)")
    p.add_argument("--chunk-fractions", default="",
                   help="comma-separated shares of a rank's tokens per sub-batch, in order (default with the "
                        "default 3 chunks at N > 1: 0.5,0.375,0.125; otherwise balanced)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-attention", action="store_true", help="skip the attention-core line")
    p.add_argument("--no-kernel-timing", action="store_true",
                   help="no per-launch events in the timed region (diagnostic; the line then lacks kernels/roofline)")
    p.add_argument("--config", type=int, default=5, choices=[1, 2, 3, 4, 5],
                   help="BASELINE config; 5 (default) is the headline, 1-4 single-GPU op chains")
    p.add_argument("--kernel", choices=KERNELS, default=None,
                   help="time one launch kind alone on --rows rows (the ncu small case)")
    p.add_argument("--rows", type=int, default=16384, help="--kernel: trie rows")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def attention_roofline(flops: float, ms: float) -> dict:
    """Roofline fields of the attention core in tree order: the path blocks
    run attention_tree_tc, whose FP32-level products are three TF32 tensor-core
    products each, so the bound is the TF32 tensor rate / 3 -- the measured
    dense bf16 rate (burst) / 2 / 3. `flops` counts the algorithmic QK and PV
    multiply-adds (2 flops each) over every (row, head, key in window)."""
    path = ROOT / "MEASURED_PEAKS.json"
    bf16, kind = 1590.0, "fallback"
    if path.exists():
        bf16, kind = float(json.loads(path.read_text())["bf16_tflops"]), "measured"
    peak = bf16 / 2 / 3
    achieved = flops / (ms * 1e-3) / 1e12
    return {"achieved": round(achieved, 2), "unit": "TFLOP/s", "bound": "tensor (3 x TF32)", "peak": round(peak, 1),
            "frac": round(achieved / peak, 3),
            "peak_kind": f"{kind} dense bf16 {bf16} TFLOP/s / 2 (TF32 rate) / 3 (TF32 products per FP32-level product)"}


# ---- clocks ----------------------------------------------------------------------------


class ClockSampler:
    """Samples this GPU's SM clock and clock-event reasons with NVML every
    100 ms while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            self._nvml = pynvml
            uuid = str(props.uuid)
            try:
                self._handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
                self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report it, never guess
            self.error = f"{type(exc).__name__}: {exc}"
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        if self._handle is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._handle is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self._handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---- distributed plumbing ----------------------------------------------------------------


def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


# ---- our arm --------------------------------------------------------------------------------


def run_ours(args):
    import torch

    from aps2026_b200 import prefill
    from aps2026_b200.prefill import ShardedPrefill, StageTimer, StandIns, Weights

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

    from aps2026_b200.shard import chunk_plan

    prompts = prefill.prompts_config5(batch=args.prompts, length=args.length)
    tokens_total = sum(len(p) for p in prompts)
    chunks = args.chunks or (1 if world == 1 else 3)
    fractions = [float(f) for f in args.chunk_fractions.split(",")] if args.chunk_fractions else None
    if fractions is None and world > 1 and chunks == 3:
        # decreasing chunks: the last chunk's gather to rank 0 is the one left
        # exposed, and 4:3:1 also computed faster than equal thirds on one
        # rank's config-5 share (15.52 vs 15.70 ms for 16,384 rows)
        fractions = [0.5, 0.375, 0.125]
    plan = chunk_plan(prompts, world, chunks, fractions)

    weights = Weights.make(dev, seed=4, layers=args.layers)
    rows = ShardedPrefill.rows_needed(prompts, plan[rank])
    free, _ = torch.cuda.mem_get_info(dev)
    set_bytes = prefill.standin_bytes(rows)
    own = rows * prefill.HIDDEN * 4 * 7 + (tokens_total * prefill.HIDDEN * 4 if rank == 0 else 0)
    pool = args.pool or int(max(1, min(args.layers, 8 if world == 1 else 32, (free * 0.8 - own) // set_bytes)))
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    t_gen = time.perf_counter()
    standins = [StandIns.make(rows, dev, gen) for _ in range(pool)]
    torch.cuda.synchronize()
    t_gen = time.perf_counter() - t_gen
    runner = ShardedPrefill(prompts, plan, weights, dev, standins, args.layers, rank=rank, exact=args.exact,
                            concurrent=not args.serial_chunks)
    stream = torch.cuda.current_stream(dev)

    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    # Inside the timed region only the dominant kernel (the fused un-permute +
    # add + LayerNorm) is bracketed by events: every event also serialises
    # its neighbouring launches, which at 8 GPUs costs ~5% of a step.
    timers = [[StageTimer(args.layers, kinds=("fused",)) for _ in runner.pipes] for _ in range(args.steps)]
    if args.no_kernel_timing:
        timers = [None] * args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        ev[0].record(stream)
        for k in range(args.steps):
            runner.step(timers[k])
            ev[k + 1].record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    ms = ev[0].elapsed_time(ev[args.steps])
    rank_ms = [ms]
    if dist:
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = ms
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        rank_ms = t.tolist()
        ms = max(rank_ms)
    ms_per_step = ms / args.steps

    # per-kernel durations: the dominant kernel from the timed region; every
    # launch kind from one fully instrumented step right after it
    bpr = prefill.bytes_per_row(args.layers)

    def summarise(timer_steps, nsteps):
        acc = {}
        for step_timers in timer_steps:
            for c, tm in enumerate(step_timers or []):
                rows_c = runner.batches[c].rows
                for kind, vals in tm.durations().items():
                    a = acc.setdefault(kind, [0, 0.0, 0.0])
                    a[0] += len(vals)
                    a[1] += sum(vals)
                    a[2] += bpr[kind if kind in bpr else "ln0"] * rows_c * len(vals)
        return {kind: dict(launches_per_step=n // nsteps, ms_per_step=round(t / nsteps, 4),
                           us_per_launch=round(t / n * 1e3, 2), gbs=round(b / (t * 1e-3) / 1e9, 1))
                for kind, (n, t, b) in acc.items()}

    timed = summarise(timers, args.steps)
    full = [[StageTimer(args.layers) for _ in runner.pipes]]
    runner.step(full[0])
    torch.cuda.synchronize()
    kern = summarise(full, 1)
    dominant = max(kern, key=lambda k: kern[k]["ms_per_step"]) if kern else None
    if dominant in timed:
        kern[dominant] = dict(timed[dominant], source="timed region")

    # e2e: host ids -> tries -> H2D -> layers -> gather -> D2H of last-token rows
    last = torch.empty((args.prompts, prefill.HIDDEN), device=dev)
    host_last = torch.empty((args.prompts, prefill.HIDDEN), pin_memory=True)

    def e2e_step():
        h2d = runner.rebuild()
        runner.step()
        if rank == 0:
            runner.last_token_rows(last)
            host_last.copy_(last, non_blocking=True)
        return h2d

    for _ in range(2):  # both pinned staging buffers in use once
        e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_steps = args.steps
    e2e_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    e2e_ev[0].record(stream)
    for _ in range(e2e_steps):
        h2d = e2e_step()
    e2e_ev[1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = e2e_ev[0].elapsed_time(e2e_ev[1]) / e2e_steps
    h2d_all = h2d
    if dist:
        t = torch.tensor([e2e_ms, float(h2d)], device=dev, dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        e2e_ms, h2d_all = float(mx[0].item()), int(t[1].item())
    d2h = host_last.numel() * 4 if rank == 0 else 0

    # the same step with the reference's reduction order (B2_FLAG_EXACT_ORDER,
    # bit-identical to the reference kernels: the mode the drop-in runs),
    # device-resident inputs, timed like `value`
    exact_line = None
    if not args.exact:
        from aps2026_b200 import ops as _ops

        for pipe in runner.pipes:
            pipe.shape.flags = _ops.B2_FLAG_EXACT_ORDER
        for _ in range(min(args.warmup, 3)):
            runner.step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        xev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        xsteps = max(1, min(args.steps, 10))
        xev[0].record(stream)
        for _ in range(xsteps):
            runner.step()
        xev[1].record(stream)
        torch.cuda.synchronize()
        x_ms = xev[0].elapsed_time(xev[1]) / xsteps
        if dist:
            t = torch.tensor([x_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            x_ms = float(t.item())
        for pipe in runner.pipes:
            pipe.shape.flags = 0
        exact_line = {"value": round(tokens_total / (x_ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(x_ms, 3),
                      "steps": xsteps, "hbm_gbs_algorithmic": round(bpr["total"] * rows * world / (x_ms / 1e3) / 1e9, 1),
                      "what": "the same step in B2_FLAG_EXACT_ORDER (the reference's serial LayerNorm sums and "
                              "exponential; bit-identical to the reference kernels), device-resident inputs"}

    # the attention core (softmax included) over this rank's trie rows, one
    # layer's worth: the one contraction between the non-GEMM ops, reported
    # beside the step (GEMM outputs are stand-ins, so it is not in the step)
    att_line = None
    if not args.no_attention:
        from aps2026_b200 import ops as _ops

        att_ms, att_keys = 0.0, 0
        for c, pipe in enumerate(runner.pipes):
            ps = runner.prompts[c]
            offs = np.zeros(len(ps) + 1, np.int32)
            offs[1:] = np.cumsum([len(p) for p in ps])
            offs_d = torch.from_numpy(offs).to(dev)
            dt = _ops.prefix_trie_device(torch.from_numpy(np.concatenate(ps).astype(np.int32)).to(dev), offs_d)
            s0 = pipe._standins[0]
            q, kv = s0.q, s0.k  # stand-ins of the chunk's q and k; k doubles as v
            out = torch.empty_like(q)
            att_keys += int(torch.clamp(dt.node_depth.long() + 1, max=_ops.SLIDING_WINDOW).sum().item())

            def launch():
                _ops.attention_tree_compact_gpu(q, kv, kv, out, dt.node_depth, dt.node_prompt, offs_d,
                                                dt.token_node, int(max(len(p) for p in ps)), dt.nodes,
                                                prefill.Q_HEADS, prefill.KV_HEADS, prefill.HEAD_DIM)
            launch()
            aev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            aev[0].record(stream)
            launch()
            aev[1].record(stream)
            launch()
            aev[2].record(stream)
            torch.cuda.synchronize()
            att_ms += min(aev[0].elapsed_time(aev[1]), aev[1].elapsed_time(aev[2]))
            del out, dt
        flops = 2 * 2 * prefill.Q_HEADS * prefill.HEAD_DIM * att_keys  # QK and PV multiply-adds per (row, key)
        att_line = {"kernel": "tc_split_kv + attention_tree_tc (tcgen05, path blocks) + attention_tree_block "
                              "(leftover blocks); compact chains, tree order",
                    "ms_per_layer": round(att_ms, 3), "flops_per_layer": flops, **attention_roofline(flops, att_ms),
                    "per_step_ms_32_layers": round(32 * att_ms, 1),
                    "what": "this rank's rows, one layer, timed after the timed region; not part of `value`"}

    clk = clocks.summary()
    allclk = [clk]
    if dist:
        allclk = [None] * world
        dist.all_gather_object(allclk, clk)

    result = None
    if rank == 0:
        peak, peak_kind = peaks()
        d = kern[dominant] if dominant else {"gbs": None}
        traffic = (round(TRAFFIC_BYTES_PER_ROW[dominant] * rows / len(runner.pipes))
                   if dominant in TRAFFIC_BYTES_PER_ROW else None)
        reasons = sorted(set(r for c in allclk for r in c.get("reasons", [])))
        mhz = [c["sm_mhz"] for c in allclk if c.get("sm_mhz")]
        tok_s = tokens_total / (ms_per_step / 1e3)
        result = {
            "metric": METRIC,
            "value": round(tok_s, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 3),
            "ms_per_step_by_rank": [round(x / args.steps, 3) for x in rank_ms],
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded token ids; GEMM outputs are seeded N(0,1) stand-ins)",
            "config": {"workload": f"config 5: {args.prompts} prompts x {args.length} tokens, {args.layers} layers, "
                                   "non-GEMM path, final hidden states gathered to rank 0",
                       "prompts": args.prompts, "tokens_per_prompt": args.length, "layers": args.layers,
                       "node_rows_per_rank": rows, "chunks_per_rank": len(runner.pipes),
                       "chunk_tokens": [runner.batches[c].tokens for c in range(len(runner.pipes))],
                       "standin_pool": pool,
                       "exact_order": args.exact,
                       "l2": "inputs larger than L2 (a step streams >= 90 GB per rank; the GEMM stand-in sets "
                             "rotate by layer, so no launch re-reads another launch's inputs)",
                       "parallelism": f"prompt shards x{world}" + (", NCCL gather to rank 0 overlapped by chunk"
                                                                  if world > 1 else "")},
            "hbm_gbs_algorithmic": round(bpr["total"] * rows * world / (ms_per_step / 1e3) / 1e9, 1),
            "roofline": {"kernel": dominant, "bound": "hbm", "achieved": d["gbs"], "peak": peak,
                         "unit": "GB/s", "frac": round(d["gbs"] / peak, 3) if d["gbs"] else None,
                         "peak_kind": peak_kind, "traffic": traffic,
                         **({"note": "chunks run concurrently on each GPU, so the kernel's events also span the "
                                     "other chunks' kernels sharing it: a lower bound on the kernel's own rate "
                                     "(its one-GPU line has one chunk); step_frac is the whole step's algorithmic "
                                     "bytes per GPU over the same peak",
                             "step_frac": round(bpr["total"] * rows / (ms_per_step / 1e3) / 1e9 / peak, 3)}
                            if runner.streams else {})},
            "kernels": kern,
            "kernels_note": "per launch kind: one fully instrumented step after the timed region; the dominant "
                            "kind (roofline) from events in the timed region" +
                            ("; chunks run concurrently, so a launch's events also span the other chunks' "
                             "kernels sharing the GPU" if runner.streams else ""),
            "clocks": {"sm_mhz": statistics.median(mhz) if mhz else None,
                       "sm_max_mhz": allclk[0].get("sm_max_mhz"), "reasons": reasons},
            "e2e": {"value": round(tokens_total / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": d2h},
            "exact_order": exact_line,
            "attention_core": att_line,
            "gpu_launches": runner.launches_per_step() * args.steps * world,
            "standin_gen_s": round(t_gen, 2),
        }
    if dist:
        runner.release()
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---- single-GPU op chains: BASELINE configs 1-4 ----------------------------------------------


def run_config(args) -> dict:
    """Configs 1-4 on one GPU, each step one pass of the config's op chain,
    L2 flushed (256 MB written) before every timed step, CUDA events around
    the chain only. Value: algorithmic GB/s (config 4: tokens/s, GB/s in
    roofline)."""
    import math

    import torch

    from aps2026_b200 import ops, prefill

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(args.config - 1)
    rn = lambda *s, std=1.0, mean=0.0: prefill._randn(s, gen, dev, mean, std)  # noqa: E731
    flush = torch.empty(64 << 20, device=dev)
    cfg = args.config
    if cfg == 1:
        x, y = rn(512, 4096), torch.empty(512, 4096, device=dev)
        w, b = rn(4096, mean=1.0, std=0.1), rn(4096, std=0.1)
        q, k = rn(512, 32 * 128), rn(512, 8 * 128)
        pos = torch.arange(512, dtype=torch.int32, device=dev)
        cos, sin = ops.rope_table_gpu(512, 128, 1e4, dev)

        def chain():
            ops.layer_norm_gpu(x, w, b, 1e-5, y, exact=args.exact)
            ops.apply_rope_tree_gpu(q, k, pos, 512, 512, 32, 8, 128, 1e4)
        nbytes, work = 38_043_648, "config 1: LayerNorm X[512,4096] + RoPE Q[512,32,128], K[512,8,128]"
        tokens = 512
    elif cfg == 2:
        H, T = 32, 2048
        scores, probs = rn(H, T, T, std=2.0), torch.empty(H, T, T, device=dev)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(128.0)))

        def chain():
            ops.causal_softmax_gpu(scores, probs, scale, 2047, exact=args.exact)
        cells = sum(min(i + 1, 2047) for i in range(T))
        nbytes = H * cells * 4 + H * T * T * 4
        work, tokens = "config 2: causal scaled softmax [32, 2048, 2048], window 2047", H * T
    elif cfg == 3:
        T = 8192
        logits = rn(T, 16)
        gu, act = rn(2 * T, 896), torch.empty(2 * T, 448, device=dev)
        eo, out = rn(2 * T, 4096), torch.empty(T, 4096, device=dev)
        routing, ws = ops.alloc_routing(T, 16, dev), ops.RouteWorkspace(T, 16, dev)

        def chain():
            ops.moe_route_gpu(logits, routing, ws)
            ops.silu_mul_gpu(gu[:, :448], gu[:, 448:], act, exact=args.exact)
            ops.moe_combine_gpu(eo, routing.routes, routing.route_positions, out)
        nbytes = (T * 16 * 4 + T * 2 + 2 * T * 4 * 2) + 2 * T * 448 * 12 + (2 * T * 4096 * 4 + T * 4096 * 4 + T * 10)
        work, tokens = "config 3: top-2 routing T=8192 + SiLU [16384, 2x448] + un-permute to [8192, 4096]", T
    else:
        prompts = prefill.prompts_config4()
        w = prefill.Weights.make(dev, 3, layers=1)
        batch = prefill.Batch.build(prompts, dev)
        sets = [prefill.StandIns.make(batch.rows, dev, gen)]
        pipe = prefill.Pipeline(batch, w, dev, exact=args.exact)
        pipe.bind_layers(sets, 1)

        def chain():
            pipe.run()
        bpr = prefill.bytes_per_row(1)
        nbytes = bpr["total"] * batch.rows
        # the attention core on the same trie rows, timed on its own (FP32
        # CUDA-core roofline): q [rows, 16, 128], k and v [rows, 4, 128]
        trie = ops.prefix_trie(prompts, with_ancestors=True)
        att_q, att_k, att_v = rn(batch.rows, 2048), rn(batch.rows, 512), rn(batch.rows, 512)
        att_o = torch.empty_like(att_q)
        att_pos = torch.from_numpy(trie.node_depth.view(np.int32)).to(dev)
        att_anc = torch.from_numpy(trie.node_anc.view(np.int32)).to(dev)
        att_keys = int(np.minimum(trie.node_depth + 1, ops.SLIDING_WINDOW).sum())
        # compact chains from the device trie (the path's own form); the dense
        # ancestor table is the reference interface's
        offs = np.zeros(len(prompts) + 1, np.int32)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        att_offs = torch.from_numpy(offs).to(dev)
        dtrie = ops.prefix_trie_device(torch.from_numpy(np.concatenate(prompts).astype(np.int32)).to(dev), att_offs)

        def attention():
            ops.attention_tree_compact_gpu(att_q, att_k, att_v, att_o, att_pos, dtrie.node_prompt, att_offs,
                                           dtrie.token_node, trie.anc_stride, batch.rows, 16, 4, 128,
                                           ops.SLIDING_WINDOW, exact=args.exact)

        def attention_dense():
            ops.attention_tree_gpu(att_q, att_k, att_v, att_o, att_pos, att_anc, trie.anc_stride, batch.rows, 16, 4,
                                   128, ops.SLIDING_WINDOW, exact=args.exact)
        work = (f"config 4: one layer's non-GEMM path, 16 prompts x 1024 tokens with a 256-token shared prefix "
                f"({batch.rows} trie rows)")
        tokens = batch.tokens
    for _ in range(args.warmup):
        chain()
    torch.cuda.synchronize()
    # The chain is captured once in a CUDA graph and replayed: at these sizes
    # (microseconds per kernel) the host's per-launch cost would otherwise
    # sit between the kernels inside the timed region.
    launch = "CUDA graph of the op chain (programmatic dependent launches kept)"
    run = chain
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                chain()
            run = graph.replay
            run()
            torch.cuda.synchronize()
        except RuntimeError as e:  # recorded in the line; the eager chain is still the GPU path
            launch = f"eager launches (graph capture failed: {str(e).splitlines()[0][:120]})"
            run = chain
    else:
        launch = "eager launches"
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        for a, b_ in ev:
            flush.zero_()
            a.record()
            run()
            b_.record()
        torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b_) for a, b_ in ev)
    att = None
    if cfg == 4:
        def time_it(fn):
            fn()
            aev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(max(3, args.steps // 4))]
            for a, b_ in aev:
                flush.zero_()
                a.record()
                fn()
                b_.record()
            torch.cuda.synchronize()
            return statistics.median(a.elapsed_time(b_) for a, b_ in aev)

        att_ms = time_it(attention)
        dense_ms = time_it(attention_dense)
        flops = 2 * 2 * 16 * 128 * att_keys  # QK and PV multiply-adds over every (row, head, key)
        kern = ("attention_tree_block (compact chains, reference order)" if args.exact else
                "tc_split_kv + attention_tree_tc (tcgen05, path blocks) + attention_tree_block (leftover blocks); "
                "compact chains, tree order")
        att = {"kernel": kern, "ms": round(att_ms, 4), "dense_table_ms": round(dense_ms, 4), "flops": flops}
        if args.exact:
            fp32_peak = 148 * 128 * 2 * 1965e6 / 1e12
            att.update({"achieved": round(flops / (att_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "bound": "fp32",
                        "peak": round(fp32_peak, 1), "frac": round(flops / (att_ms * 1e-3) / 1e12 / fp32_peak, 3),
                        "peak_kind": "nominal FP32 CUDA-core rate (148 SMs x 128 lanes x 2 flops x 1965 MHz); "
                                     "MEASURED_PEAKS.json has no FP32 figure"})
        else:
            att.update(attention_roofline(flops, att_ms))
    peak, peak_kind = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    res = {"metric": f"config {cfg} " + ("non-GEMM tokens/s" if cfg == 4 else "algorithmic HBM GB/s"),
           "value": round(tokens / (ms * 1e-3), 1) if cfg == 4 else round(gbs, 1),
           "unit": "tokens/s" if cfg == 4 else "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic (seeded)",
           "config": {"workload": work, "algorithmic_bytes": nbytes, "exact_order": args.exact,
                      "l2": "flushed (256 MB written) before every timed step", "launch": launch},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 3), "peak_kind": peak_kind, "traffic": None},
           "clocks": {k: v for k, v in clocks.summary().items() if k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    if att:
        res["attention_core"] = att
    return res


# ---- one kernel on its own ---------------------------------------------------------------------

KERNELS = ("ln", "add_ln", "fused", "rope", "silu", "combine", "gather", "route")


def run_kernel(args) -> dict:
    """One launch kind of the path alone on `--rows` trie rows at the
    config.h shapes (hidden 4096, 16 / 4 heads of 128, 16 experts,
    intermediate 448): L2 flushed (256 MB written) before each timed launch,
    CUDA events around the launch on its stream, median over `--steps`.
    Value: algorithmic GB/s (each tensor read or written once). This is the
    small case the ncu summaries are captured on."""
    import torch

    from aps2026_b200 import ops, prefill as P

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    R, H = args.rows, P.HIDDEN
    gen = torch.Generator(device=dev).manual_seed(11)
    rn = lambda *s, std=1.0, mean=0.0: P._randn(s, gen, dev, mean, std)  # noqa: E731
    emp = lambda *s: torch.empty(s, device=dev)  # noqa: E731
    gamma, beta = rn(H, mean=1.0, std=0.1), rn(H, std=0.1)
    flush = torch.empty(64 << 20, device=dev)
    kind, exact = args.kernel, args.exact
    if kind in ("fused", "combine"):
        routing = ops.moe_route_gpu(rn(R, P.EXPERTS))
    if kind == "ln":
        x, y = rn(R, H), emp(R, H)
        fn = lambda: ops.layer_norm_gpu(x, gamma, beta, 1e-5, y, exact=exact)  # noqa: E731
        nbytes = 2 * R * H * 4 + 2 * H * 4
    elif kind == "add_ln":
        x, res, y = rn(R, H), rn(R, H), emp(R, H)
        fn = lambda: ops.add_layer_norm_gpu(x, res, gamma, beta, 1e-5, y, exact=exact)  # noqa: E731
        nbytes = 4 * R * H * 4 + 2 * H * 4
    elif kind == "fused":
        eo, carry, xo, y = rn(2 * R, H), rn(R, H), emp(R, H), emp(R, H)
        fn = lambda: ops.moe_combine_add_layer_norm_gpu(eo, routing.routes, routing.route_positions, carry,  # noqa
                                                        gamma, beta, 1e-5, xo, y, exact=exact)
        nbytes = P.bytes_per_row(1)["fused"] * R + 2 * H * 4
    elif kind == "rope":
        q, k = rn(R, P.Q_HEADS * P.HEAD_DIM), rn(R, P.KV_HEADS * P.HEAD_DIM)
        pos = (torch.arange(R, dtype=torch.int32, device=dev) % 2048).contiguous()
        fn = lambda: ops.apply_rope_tree_gpu(q, k, pos, R, 2048, P.Q_HEADS, P.KV_HEADS, P.HEAD_DIM, 1e4)  # noqa
        nbytes = P.bytes_per_row(1)["rope"] * R
    elif kind == "silu":
        gu, act = rn(2 * R, 2 * P.INTER), emp(2 * R, P.INTER)
        fn = lambda: ops.silu_mul_gpu(gu[:, :P.INTER], gu[:, P.INTER:], act, exact=exact)  # noqa: E731
        nbytes = P.bytes_per_row(1)["silu"] * R
    elif kind == "combine":
        eo, out = rn(2 * R, H), emp(R, H)
        fn = lambda: ops.moe_combine_gpu(eo, routing.routes, routing.route_positions, out)  # noqa: E731
        nbytes = 3 * R * H * 4 + R * (2 + 8)
    elif kind == "gather":
        emb, out = rn(P.VOCAB, H, std=0.02), emp(R, H)
        ids = torch.randint(0, P.VOCAB, (R,), generator=gen, device=dev, dtype=torch.int32)
        fn = lambda: ops.gather_rows_gpu(emb, ids, out)  # noqa: E731
        nbytes = 2 * R * H * 4 + 4 * R
    else:  # route
        logits = rn(R, P.EXPERTS)
        rt, ws = ops.alloc_routing(R, P.EXPERTS, dev), ops.RouteWorkspace(R, P.EXPERTS, dev)
        fn = lambda: ops.moe_route_gpu(logits, rt, ws)  # noqa: E731
        nbytes = P.bytes_per_row(1)["route"] * R
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        for a, b_ in ev:
            flush.zero_()
            a.record()
            fn()
            b_.record()
        torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b_) for a, b_ in ev)
    peak, peak_kind = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"metric": f"kernel {kind} algorithmic HBM GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": f"{kind} on {R} rows (hidden {H})", "rows": R, "algorithmic_bytes": nbytes,
                       "exact_order": exact, "l2": "flushed (256 MB written) before every timed launch"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 3), "peak_kind": peak_kind, "traffic": None},
            "clocks": {k: v for k, v in clocks.summary().items() if k in ("sm_mhz", "sm_max_mhz", "reasons")}}


# ---- CPU baseline / reference arm ---------------------------------------------------------


def cpu_sample_inputs(rows: int, seed: int = 7):
    """Host stand-ins for a bounded CPU sample of the same workload."""
    from aps2026_b200 import prefill as P

    g = np.random.default_rng(seed)
    n = lambda *s: g.standard_normal(s, dtype=np.float32)  # noqa: E731
    # the sample gathers `rows` embedding rows; a table of `rows` rows suffices
    prompts = [g.integers(0, rows, 2048).astype(np.int32) for _ in range(rows // 2048)]
    emb = (n(rows, P.HIDDEN) * 0.02).astype(np.float32)
    s = dict(q=n(rows, P.Q_HEADS * P.HEAD_DIM), k=n(rows, P.KV_HEADS * P.HEAD_DIM), attn=n(rows, P.HIDDEN),
             logits=n(rows, P.EXPERTS), gate_up=n(2 * rows, 2 * P.INTER), expert_out=n(2 * rows, P.HIDDEN))
    ln = [(1 + 0.1 * n(P.HIDDEN), 0.1 * n(P.HIDDEN)) for _ in range(2)]
    return prompts, emb, s, ln


def cpu_baseline_port(rows: int = 8192, budget_s: float = 10.0) -> dict:
    """The CPU oracle (a restatement of the reference kernels, OpenMP on all
    host threads) over a bounded sample: one-layer passes of the pipeline
    (gather, layer, final add + LN) on `rows` rows, repeated until about
    `budget_s` seconds; tokens/s scaled to the 32-layer path."""
    import oracle

    prompts, emb, s, ln = cpu_sample_inputs(rows)
    trie = oracle.prefix_trie(prompts, with_ancestors=False)
    passes, t = 0, 0.0
    while t < budget_s and passes < 32:
        t0 = time.perf_counter()
        oracle.prefill_layers(emb, trie["node_token"], trie["node_depth"], [s], [ln[0]], [ln[1]], ln[0], 1)
        t += time.perf_counter() - t0
        passes += 1
    return {"value": round(rows * passes / 32 / t, 1), "unit": "tokens/s", "cores": oracle.num_threads(),
            "cpu_model": cpu_model(), "kind": "port",
            "sample": f"oracle pipeline, {passes} one-layer passes over {rows} rows (gather + layer + final LN), "
                      f"{t:.1f} s, scaled to 32 layers"}


def reference_layer(rows: int, s, ln, emb, node_token, node_depth, lens) -> float:
    """One decoder layer's non-GEMM path on the CPU through the reference's
    own host ops (oracle/_ref: tensor_ops::layer_norm, apply_rope, add_inplace,
    silu + mul, as PhiDecoderLayer::forward's CPU branch calls them,
    src/layer.cu:302-326); the top-2 routing and the expert un-permute, whose
    reference CPU code is private to PhiMoE (src/layer.cu:69-92, :123-147),
    run through the oracle's restatement. Returns seconds of op time."""
    import ctypes as C

    import oracle

    r = oracle.ref()
    sec = C.c_double()
    total = 0.0
    from aps2026_b200 import prefill as P

    h = P.HIDDEN
    t0 = time.perf_counter()
    x = oracle.gather_rows(emb, node_token)
    total += time.perf_counter() - t0
    normed = np.empty_like(x)
    r.ref_cpu_layer_norm(x.ctypes.data, ln[0][0].ctypes.data, ln[0][1].ctypes.data, normed.ctypes.data, rows, h,
                         1e-5, C.addressof(sec))
    total += sec.value
    lens_arr = np.asarray(lens, dtype=np.uint64)
    r.ref_cpu_apply_rope(s["q"].ctypes.data, s["k"].ctypes.data, lens_arr.ctypes.data, len(lens), P.Q_HEADS,
                         P.KV_HEADS, P.HEAD_DIM, 1e4, C.addressof(sec))
    total += sec.value
    attn = s["attn"]
    r.ref_cpu_add_inplace(attn.ctypes.data, x.ctypes.data, attn.size, C.addressof(sec))
    total += sec.value
    post = np.empty_like(attn)
    r.ref_cpu_layer_norm(attn.ctypes.data, ln[1][0].ctypes.data, ln[1][1].ctypes.data, post.ctypes.data, rows, h,
                         1e-5, C.addressof(sec))
    total += sec.value
    t0 = time.perf_counter()
    route = oracle.moe_route(s["logits"])
    total += time.perf_counter() - t0
    gate = np.ascontiguousarray(s["gate_up"][:, :P.INTER])
    up = np.ascontiguousarray(s["gate_up"][:, P.INTER:])
    act = np.empty_like(gate)
    r.ref_cpu_silu_mul(gate.ctypes.data, up.ctypes.data, act.ctypes.data, gate.size, C.addressof(sec))
    total += sec.value
    t0 = time.perf_counter()
    ff = oracle.moe_combine(s["expert_out"], route["routes"], route["route_positions"], rows)
    total += time.perf_counter() - t0
    r.ref_cpu_add_inplace(ff.ctypes.data, attn.ctypes.data, ff.size, C.addressof(sec))
    total += sec.value
    return total


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_gpu_kernels(rows: int, layers: int, steps: int) -> dict:
    """The reference's own non-GEMM kernels (src/tensor.cu, compiled from its
    source into oracle/_ref/libref.so) on this GPU, for comparison with ours
    on the same hardware: one decoder layer's sequence as forward_carry
    launches it (k_add_layer_norm for the carried add + input LayerNorm,
    k_rope on Q then K, k_add_layer_norm after attention, the routing
    kernels, k_silu_mul, k_moe_combine) on `rows` rows with seeded stand-ins,
    timed per kernel with CUDA events (median of `steps`), scaled to
    `layers` layers plus the embedding gather and the final add + LN."""
    import ctypes as C

    import torch

    import oracle
    from aps2026_b200 import ops, prefill as P

    r = oracle.ref()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(12)
    rn = lambda *s, std=1.0, mean=0.0: P._randn(s, gen, dev, mean, std)  # noqa: E731
    emp = lambda *s, dt=torch.float32: torch.empty(s, device=dev, dtype=dt)  # noqa: E731
    H, s = P.HIDDEN, torch.cuda.current_stream().cuda_stream
    x, carry, y = rn(rows, H), rn(rows, H), emp(rows, H)
    w, b = rn(H, mean=1.0, std=0.1), rn(H, std=0.1)
    q, k = rn(rows, P.Q_HEADS * P.HEAD_DIM), rn(rows, P.KV_HEADS * P.HEAD_DIM)
    pos = (torch.arange(rows, dtype=torch.int32, device=dev) % 2048).contiguous()
    cos, sin = ops.rope_table_gpu(2048, P.HEAD_DIM, 1e4, dev)
    logits = rn(rows, P.EXPERTS)
    n64, n128 = ops.queue_lengths(rows, P.EXPERTS)
    rt = [emp(2 * rows, dt=torch.uint8), emp(P.EXPERTS, dt=torch.int32), emp(P.EXPERTS + 1, dt=torch.int32),
          emp(2 * rows, dt=torch.int32), emp(2 * rows, dt=torch.int32), emp(n64, dt=torch.int32),
          emp(n64, dt=torch.int32), emp(n128, dt=torch.int32), emp(n128, dt=torch.int32)]
    gate, up, act = rn(2 * rows, P.INTER), rn(2 * rows, P.INTER), emp(2 * rows, P.INTER)
    eo, out = rn(2 * rows, H), emp(rows, H)
    emb = rn(P.VOCAB, H, std=0.02)
    ids = torch.randint(0, P.VOCAB, (rows,), generator=gen, device=dev, dtype=torch.int32)
    flush = torch.empty(64 << 20, device=dev)
    pp = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    launch = {
        "add_ln": lambda: r.ref_k_add_layer_norm(pp(x), pp(carry), pp(w), pp(b), pp(y), rows, H, 1e-5, s),
        "rope": lambda: r.ref_k_rope(pp(q), pp(k), pp(pos), pp(cos), pp(sin), rows, P.Q_HEADS, P.KV_HEADS,
                                     P.HEAD_DIM, s),
        "route": lambda: r.ref_k_moe_route(pp(logits), rows, *[pp(t) for t in rt], s),
        "silu": lambda: r.ref_k_silu_mul(pp(gate), pp(up), pp(act), 2 * rows * P.INTER, s),
        "combine": lambda: r.ref_k_moe_combine(pp(eo), pp(rt[0]), pp(rt[4]), pp(out), rows, H, s),
        "gather": lambda: r.ref_k_gather_rows(pp(emb), pp(ids), pp(out), rows, H, s),
    }
    ms = {}
    for name, fn in launch.items():
        if fn() != 0:
            raise RuntimeError(f"reference kernel {name} failed to launch")
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, e in ev:
            flush.zero_()
            a.record()
            fn()
            e.record()
        torch.cuda.synchronize()
        ms[name] = statistics.median(a.elapsed_time(e) for a, e in ev)
    layer = 2 * ms["add_ln"] + ms["rope"] + ms["route"] + ms["silu"] + ms["combine"]
    step = layers * layer + ms["gather"] + ms["add_ln"]
    return {"value": round(rows / (step * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(step, 3),
            "layer_ms": {k: round(v, 4) for k, v in ms.items()}, "rows": rows,
            "what": f"the reference's own kernels (oracle/_ref/libref.so, src/tensor.cu built for sm_100a) on "
                    f"{torch.cuda.get_device_name(dev)}: one layer on {rows} rows timed per kernel (median of "
                    f"{steps}, L2 flushed), x {layers} layers + gather + final add-LN; k_silu_mul stands for the "
                    f"SiLU epilogue the reference fuses into its expert GEMM"}


def run_reference(args):
    import oracle

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if not oracle.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libref.so (the reference built from its source) "
                                                    "is missing; build it with `make -C oracle` where the "
                                                    "reference tree exists"}
    # One step of this arm = one bounded sample of the workload: one decoder
    # layer's non-GEMM path over `rows` rows on the host cores. value scales
    # its rate to the whole workload (layers x tokens), flagged extrapolated.
    rows = 2048
    prompts, emb, s, ln = cpu_sample_inputs(rows, seed=8)
    trie = oracle.prefix_trie(prompts, with_ancestors=False)
    lens = [len(p) for p in prompts]
    base = {k: v.copy() for k, v in s.items()}
    for _ in range(args.warmup):
        reference_layer(rows, {k: v.copy() for k, v in base.items()}, ln, emb, trie["node_token"],
                        trie["node_depth"], lens)
    secs = []
    for _ in range(args.steps):
        secs.append(reference_layer(rows, {k: v.copy() for k, v in base.items()}, ln, emb, trie["node_token"],
                                    trie["node_depth"], lens))
    t_layer = statistics.mean(secs)
    tokens_total = args.prompts * args.length
    scale = args.layers * tokens_total / rows
    value = tokens_total / (t_layer * scale)
    sample = (f"one step = one decoder layer's non-GEMM path on {rows} rows: reference host ops (oracle/_ref) for "
              f"LN / RoPE / add / SiLU*mul, oracle port for routing and un-permute (the reference's are private "
              f"to PhiMoE); {t_layer:.3f} s per step, value scaled x{scale:g} to {args.layers} layers x "
              f"{tokens_total} tokens")
    res = {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_layer * 1e3, 3),
           "step_is": f"a bounded sample: one layer on {rows} rows", "extrapolated": True,
           "scale_to_workload": scale,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": {"workload": f"config 5: {args.prompts} prompts x {args.length} tokens, "
                                                       f"{args.layers} layers, non-GEMM path (CPU sample)"},
           "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": oracle.num_threads(),
                            "cpu_model": cpu_model(), "kind": "reference", "sample": sample},
           "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    try:
        import torch

        if torch.cuda.is_available():
            res["reference_gpu_kernels"] = reference_gpu_kernels(args.prompts * args.length, args.layers, 5)
    except Exception as exc:  # informational only; the arm's value is the CPU path
        res["reference_gpu_kernels"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    return res


def main():
    args = parse()
    if args.impl == "reference":
        res = run_reference(args)
        if res is not None:
            print(json.dumps(res))
        return
    if args.kernel:
        print(json.dumps(run_kernel(args)))
        return
    if args.config != 5:
        print(json.dumps(run_config(args)))
        return
    res = run_ours(args)
    if res is not None:
        if args.gpus == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_port()
        print(json.dumps(res))


if __name__ == "__main__":
    main()
