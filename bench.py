"""Benchmark: paged-attention decode tokens/s (+ HBM GB/s) on B200.

One step = append one token per sequence through the slot mapping, then decode
every sequence over ctx+1 tokens (one call of the fused C-ABI entry point).
Default workload: configuration c2 (Llama-7B-shaped, f32 KV, batch 64, 32
heads x 128, block 16, context 2048, 16384-block pool).  Under torchrun the
64 sequences shard over the N GPUs with distribute_batch's contiguous split
(strong scaling: each GPU owns its sequences' blocks in its own pool; no
data-path collective).  `--weak` gives every rank a full replica instead.
After the headline, configurations c3, c4, c5 are measured at the same N in
the same run (`per_config`): c3/c5 sharded by attended tokens, c4 split by
KV heads with one NCCL all-gather of the outputs on N > 1.  Inputs exceed
the 126 MB L2 (c2 4.3 GB of KV per step), so no flush is needed between
steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2]
  python bench.py --impl reference ...   # CPU arm (the oracle port)
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn decode tokens/s"

# DRAM bytes (read + write) per decode launch of the 1-GPU workload, from
# earlier full-size ncu captures of the decode kernel (the committed profile
# summaries).  Reported as roofline.traffic next to the algorithmic bytes;
# None where no full-size capture exists.
TRAFFIC_MEASURED = {"c2": 4334.7e6, "c3": 694.3e6}


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.index, self.samples, self.reasons, self.stop = index, [], set(), threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
        self.t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self.stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.nv:
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.nv:
            self.t.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def host_sample_case(spec, n_seqs: int, seed: int = 1, with_append: bool = False):
    """A CPU-side case with the shapes and value distributions of `spec` for
    `n_seqs` sequences (a pool of exactly the blocks they use), drawn with
    numpy on the host (timing input only; nothing is compared).  Returns
    (layout, (k_cache, v_cache, block_tables, ctx + 1, q[, k_new, v_new,
    slots])) as numpy arrays (16-bit types as bit patterns)."""
    import numpy as np
    from dataclasses import replace

    import torch

    import oracle
    from clove_b200.workload import make_layout
    lay = make_layout(replace(spec, num_blocks=0, tables="permutation"), seed=spec.seed + seed, batch=n_seqs)
    rng = np.random.default_rng(spec.seed + seed)
    f32 = spec.dtype == torch.float32
    # one 16 Mi-element block of N(0,1) draws, tiled (CPU timing input only;
    # drawing every element costs more than the timed steps on large pools)
    src = rng.standard_normal(1 << 24, dtype=np.float32)

    def draw(shape, scale=1.0):
        x = np.empty(shape, np.float32)
        flat = x.reshape(-1)
        step = src.size
        for i in range(0, flat.size, step):
            n = min(step, flat.size - i)
            flat[i:i + n] = src[:n]
        if scale != 1.0:
            x *= np.float32(scale)
        if f32:
            return x
        if spec.dtype == torch.float16:
            return x.astype(np.float16).view(np.uint16)
        u = x.view(np.uint32)  # bf16, round to nearest even
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    row = (spec.block_size, spec.num_kv_heads, spec.head_dim)
    kc = draw((lay.num_blocks,) + row, spec.kv_scale)
    vc = draw((lay.num_blocks,) + row, spec.kv_scale)
    q = draw((lay.batch, spec.num_q_heads, spec.head_dim))
    case = (kc, vc, lay.block_tables, (lay.context_lens + 1).astype(np.int32), q)
    if with_append:
        slots = oracle.append_slots(lay.block_tables, lay.context_lens, spec.block_size)
        kn = draw((lay.batch, spec.num_kv_heads, spec.head_dim), spec.kv_scale)
        vn = draw((lay.batch, spec.num_kv_heads, spec.head_dim), spec.kv_scale)
        case = case + (kn, vn, slots)
    return lay, case


def cpu_arm(lay, case, budget_s: float, max_reps: int | None = None) -> dict:
    """Time the oracle's f32 restatement (reference CPU idiom) on the host
    cores over the sampled sequences, repeated for about `budget_s` seconds."""
    import numpy as np

    import oracle
    from clove_b200.workload import dtype_code
    kc, vc, bt, ctx, qs = case
    threads = os.cpu_count() or 1
    code = dtype_code(lay.spec.dtype)
    scale = 1.0 / np.sqrt(lay.spec.head_dim)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.decode_f32(code, qs, kc, vc, bt, ctx, scale, nthreads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or (max_reps and reps >= max_reps):
            break
    seqs = ctx.shape[0]
    return {"value": seqs * reps / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} sequences shaped like config {lay.spec.name} (ctx+1 = "
                      f"{int(ctx.min())}..{int(ctx.max())}), decode only, {reps} reps in {el:.1f} s"}


def _dist():
    import torch
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        torch.cuda.set_device(local) if torch.cuda.is_available() else None
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    return ws, rank, local


def run_reference(args) -> None:
    """CPU arm: the oracle port of the reference's CPU idiom (slot-mapping
    append + f32 decode) on all host cores, rank 0 only.  A step is the
    configured workload's whole batch when (steps + warmup) such steps fit
    in about 150 s, else the first n sequences of it (n >= 8)."""
    import numpy as np

    import oracle
    from clove_b200.workload import CONFIGS, dtype_code

    ws, rank, _ = _dist()
    if rank != 0:
        return
    spec = CONFIGS[args.config]
    lay, case = host_sample_case(spec, spec.batch if args.batch is None else args.batch, with_append=True)
    kc, vc, bt, ctx, qs, kn, vn, slots = case
    threads = os.cpu_count() or 1
    code = dtype_code(spec.dtype)
    scale = 1.0 / np.sqrt(spec.head_dim)

    def step(n):
        oracle.reshape_and_cache(kc, vc, kn[:n], vn[:n], slots[:n])
        oracle.decode_f32(code, qs[:n], kc, vc, bt[:n], ctx[:n], scale, nthreads=threads)

    n = lay.batch
    t0 = time.perf_counter()
    step(n)
    t1 = time.perf_counter() - t0
    budget = 150.0
    if (args.steps + args.warmup) * t1 > budget:
        n = max(8, min(n, int(n * budget / ((args.steps + args.warmup) * t1))))
    for _ in range(max(args.warmup - 1, 0)):
        step(n)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(n)
    el = time.perf_counter() - t0
    val = n * args.steps / el
    cb = {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
          "sample": f"per step {n} of the {lay.batch} sequences of config {spec.name} (ctx+1 = "
                    f"{int(ctx[:n].min())}..{int(ctx[:n].max())}): slot-mapping append + f32 decode, "
                    f"oracle restatement of the reference's CPU idiom on {threads} host threads"}
    print(json.dumps({"metric": METRIC, "value": val, "unit": "tokens/s", "impl": "reference", "n_gpus": ws,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                      "dtype": _dtype_name(spec.dtype), "data": "synthetic",
                      "config": headline_config(args.config, ws, args.weak, args.batch),
                      "cpu_baseline": cb,
                      "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def _head_gather() -> str:
    """Output exchange of the c4 KV-head split: "nccl" (all_gather_into_tensor,
    default: the faster whole step at 2 GPUs) or "peer" (the library's P2P
    store kernel over NVLink); CLOVE_HEAD_GATHER selects."""
    g = os.environ.get("CLOVE_HEAD_GATHER", "nccl")
    if g not in ("peer", "nccl"):
        raise ValueError(f"CLOVE_HEAD_GATHER={g!r}: expected peer or nccl")
    return g


def _partition(mode: str, name: str, ws: int) -> str:
    return {"heads": f"kv-heads/{ws} + all-gather of outputs ({_head_gather()})",
            "sequences": (f"sequences sharded over {ws} GPUs ({_policy(name)}), own pool per GPU, no collective")
            if ws > 1 else "1 GPU",
            "replica": f"{ws} independent full replicas"}[mode]


def headline_config(name: str, ws: int, weak: bool, batch=None) -> dict:
    """The `config` object of the headline line (both arms), from host-side
    layout metadata only."""
    from dataclasses import replace

    from clove_b200.workload import CONFIGS, make_layout, shard_layout
    spec = CONFIGS[name]
    if batch is not None:
        spec = replace(spec, num_blocks=0)
    if name == "c4" and ws > 1:
        mode, lay = "heads", make_layout(spec, batch=batch)
        gb, kv = lay.batch, lay.kv_bytes()
    elif weak and ws > 1:
        mode, lay = "replica", make_layout(spec, batch=batch)
        gb, kv = lay.batch * ws, lay.kv_bytes() * ws
    else:
        mode = "sequences"
        lay, _ = shard_layout(spec, ws, 0, batch=batch)
        gb, kv = lay.extra.get("global_batch", lay.batch), lay.extra.get("global_kv_bytes", lay.kv_bytes())
    return {"workload": spec.name, "description": spec.description, "batch_per_gpu": lay.batch,
            "global_batch": gb, "num_q_heads": spec.num_q_heads, "num_kv_heads": spec.num_kv_heads,
            "head_dim": spec.head_dim, "block_size": spec.block_size, "num_blocks_per_gpu": lay.num_blocks,
            "kv_bytes_per_step": kv, "l2": "inputs larger than L2 (no flush)",
            "parallelism": _partition(mode, name, ws)}


def _dtype_name(dt) -> str:
    import torch
    return {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[dt]


class DecodeCase:
    """One configuration's decode step on this rank: its pool, inputs and a
    `step()` that launches append + decode (+ the output all-gather under KV
    -head sharding) on the current stream."""

    def __init__(self, name: str, ws: int, rank: int, dev, batch=None, weak: bool = False):
        from dataclasses import replace

        import torch

        from clove_b200 import KVPool
        from clove_b200.distributed import head_sharded_append_decode
        from clove_b200.workload import CONFIGS, fill_values, make_layout, shard_layout

        spec = CONFIGS[name]
        if batch is not None:
            spec = replace(spec, num_blocks=0)  # pool sized to the blocks used (profiling)
        self.spec, self.ws, self.rank, self.dev = spec, ws, rank, dev
        # c4 on N > 1 GPUs: KV heads split across ranks + one all-gather of
        # the outputs.  Every other configuration on N > 1 GPUs: the global
        # batch sharded by sequence (own pool and tables per rank, no
        # collective); --weak gives every rank a full replica instead.
        self.head_split = name == "c4" and ws > 1
        self.mode = "heads" if self.head_split else ("replica" if weak and ws > 1 else "sequences")
        if self.head_split:
            lay = make_layout(spec, seed=spec.seed, batch=batch)  # same tables on every rank
            lspec = replace(spec, num_kv_heads=spec.num_kv_heads // ws, num_q_heads=spec.num_q_heads // ws,
                            seed=spec.seed + rank)
            llay = replace(lay, spec=lspec, seed=lspec.seed)
            self.pool = KVPool(lay.num_blocks, spec.block_size, lspec.num_kv_heads, spec.head_dim, spec.dtype, dev)
            _, kn, vn, _ = fill_values(llay, dev, self.pool.storage)
            gq = torch.Generator(device=dev)
            gq.manual_seed(spec.seed)
            q_all = torch.randn((lay.batch, spec.num_q_heads, spec.head_dim), generator=gq, device=dev).to(spec.dtype)
            hl = spec.num_q_heads // ws
            q = q_all[:, rank * hl:(rank + 1) * hl].contiguous()  # this rank's query heads
            self.gbuf = torch.empty((ws * lay.batch, hl, spec.head_dim), dtype=torch.float32, device=dev)
            if _head_gather() == "peer":
                from clove_b200.distributed import PeerGather
                self.peer = PeerGather(lay.batch * hl * spec.head_dim * 4, dev)
            self.global_batch = lay.batch
            self.kv_local = lay.kv_bytes() // ws
            self.kv_total = lay.kv_bytes()
        else:
            if self.mode == "replica":
                lay = make_layout(spec, seed=spec.seed + rank, batch=batch)
                self.global_batch = lay.batch * ws
                self.kv_total = lay.kv_bytes() * ws
            else:
                lay, _ = shard_layout(spec, ws, rank, batch=batch)
                self.global_batch = lay.extra.get("global_batch", lay.batch)
                self.kv_total = lay.extra.get("global_kv_bytes", lay.kv_bytes())
            self.kv_local = lay.kv_bytes()
            self.pool = KVPool(lay.num_blocks, spec.block_size, spec.num_kv_heads, spec.head_dim, spec.dtype, dev)
            q, kn, vn, _ = fill_values(lay, dev, self.pool.storage)
        self.lay, self.q, self.kn, self.vn = lay, q, kn, vn
        self.bt = torch.from_numpy(lay.block_tables).to(dev)
        self.cl = torch.from_numpy(lay.context_lens).to(dev)
        self.out = torch.empty((lay.batch, q.shape[1], spec.head_dim), dtype=torch.float32, device=dev)
        self.max_ctx = lay.max_ctx
        self._hs = head_sharded_append_decode
        if not hasattr(self, "peer"):
            self.peer = None

    def decode(self):
        return self.pool.append_decode(self.q, self.kn, self.vn, self.bt, self.cl, max_ctx=self.max_ctx, out=self.out)

    def gather(self):
        import torch.distributed as dist
        if self.peer is not None:
            self.peer(self.out, self.gbuf)
        else:
            dist.all_gather_into_tensor(self.gbuf, self.out)

    def step(self):
        self.decode()
        if self.head_split:
            self.gather()

    def close(self):
        if self.peer is not None:
            self.peer.close()
        self.pool.close()


def _max_over_ranks(x: float, ws: int, dev) -> float:
    import torch
    import torch.distributed as dist
    if ws <= 1:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws: int) -> None:
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def time_case(case: DecodeCase, steps: int, warmup: int, graph: bool = True, local: int = 0):
    """Warm up, capture one step in a CUDA graph, and time `steps` replays
    with CUDA events (barrier + synchronize on both sides).  Returns
    (ms per step on this rank, max over ranks, launches per step, clocks)."""
    import torch

    from clove_b200 import launch_count
    for _ in range(max(warmup, 3)):
        case.step()
    torch.cuda.synchronize()
    if case.pool.decode_status(case.lay.batch, case.q.shape[1], case.max_ctx) != 0:
        raise RuntimeError(f"device check flags raised on the {case.spec.name} workload")
    n0 = launch_count()
    case.step()
    torch.cuda.synchronize()
    per_step = launch_count() - n0
    run = case.step
    if graph:
        # the timed region then holds only device work (plan, decode,
        # combine, and the all-gather under head sharding), not Python
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            case.step()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    stream = torch.cuda.current_stream(case.dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(case.ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(steps):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
    _barrier(case.ws)
    ms = ev0.elapsed_time(ev1) / steps
    return ms, _max_over_ranks(ms, case.ws, case.dev), per_step, clocks.summary()


def phase_breakdown(case: DecodeCase, reps: int = 20) -> dict:
    """Per-launch device times of one step, from CUDA events around each
    launch (eager, serialised: the programmatic overlap of the plan ->
    decode -> combine chain is lost, as in a profiler's launch list), the
    median over `reps` steps, max over ranks."""
    import ctypes as C

    import torch

    from clove_b200 import _lib
    L = _lib.lib()
    stream = torch.cuda.current_stream(case.dev)
    rows = []
    L.clove_cuda_debug_phase_timing(1)
    try:
        for _ in range(reps + 2):
            case.decode()
            pl, de, co = C.c_float(), C.c_float(), C.c_float()
            _lib.check(L.clove_cuda_debug_phase_ms(C.byref(pl), C.byref(de), C.byref(co)))
            ag = 0.0
            if case.head_split:
                _barrier(case.ws)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                case.gather()
                e1.record(stream)
                e1.synchronize()
                ag = e0.elapsed_time(e1)
            rows.append((pl.value, de.value, co.value, ag))
    finally:
        L.clove_cuda_debug_phase_timing(0)
    rows = rows[2:]
    med = [statistics.median(r[i] for r in rows) for i in range(4)]
    med = [_max_over_ranks(x, case.ws, case.dev) for x in med]
    out = {"plan_ms": med[0], "decode_ms": med[1], "combine_ms": med[2]}
    if case.head_split:
        out["all_gather_ms"] = med[3]
    out["note"] = "CUDA events around each launch, eager and serialised (median of %d steps, max over ranks)" % reps
    return out


def config_record(case: DecodeCase, ms_max: float, peak: float, launches: int | None = None) -> dict:
    ws = case.ws
    # KV bytes per GPU per step at the job's step time (slowest rank)
    achieved = case.kv_total / ws / (ms_max * 1e-3) / 1e9
    rec = {"value": case.global_batch / (ms_max * 1e-3), "unit": "tokens/s", "ms_per_step": ms_max,
           "hbm_gbs": achieved, "global_batch": case.global_batch, "batch_per_gpu": case.lay.batch,
           "kv_bytes_per_step": case.kv_total, "dtype": _dtype_name(case.spec.dtype),
           "partition": _partition(case.mode, case.spec.name, ws),
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak}}
    if launches is not None:
        rec["gpu_launches_per_step"] = launches
    return rec


def _policy(name: str) -> str:
    from clove_b200.workload import SHARD_POLICY
    return {"contiguous": "distribute_batch contiguous split", "tokens": "token-balanced"}[
        SHARD_POLICY.get(name, "contiguous")]


def run_ours(args) -> None:
    import gc

    import torch

    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, peak_kind = _peaks()

    # ---- headline: the configured workload (c2 by default) ----
    case = DecodeCase(args.config, ws, rank, dev, batch=args.batch, weak=args.weak)
    spec, lay = case.spec, case.lay
    ms, ms_max, per_step, clocks = time_case(case, args.steps, args.warmup, graph=not args.no_graph, local=local)
    launches = per_step * args.steps
    breakdown = phase_breakdown(case)

    # ---- end to end: host (pinned) inputs -> device -> result back to host ----
    hq = case.q.cpu().pin_memory()
    hk, hv = case.kn.cpu().pin_memory(), case.vn.cpu().pin_memory()
    hbt, hcl = case.bt.cpu().pin_memory(), case.cl.cpu().pin_memory()
    out = case.out
    hout = torch.empty((lay.batch, ws, out.shape[1], spec.head_dim) if case.head_split else out.shape,
                       dtype=torch.float32).pin_memory()
    dq, dk, dv, dbt, dcl = (torch.empty_like(x, device=dev) for x in (hq, hk, hv, hbt, hcl))
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hbt, hcl))
    d2h = hout.numel() * 4
    stream = torch.cuda.current_stream(dev)

    if case.head_split:
        def e2e_step():
            for d, h in ((dq, hq), (dk, hk), (dv, hv), (dbt, hbt), (dcl, hcl)):
                d.copy_(h, non_blocking=True)
            res = case._hs(case.pool, dq, dk, dv, dbt, dcl, ws, case.max_ctx, out_local=out, gather_buf=case.gbuf,
                           peer=case.peer)
            hout.copy_(res, non_blocking=True)
    else:
        # Through the reference-facing FFI (include/clove_ffi.h): tensors made
        # from host buffers, clove_paged_attention, result copied back to host.
        import ctypes as C

        from clove_b200 import _lib
        L = _lib.lib()
        code = {torch.float32: 0, torch.bfloat16: 160, torch.float16: 16}[spec.dtype]

        def mk(t, dt):
            shp = (C.c_int64 * t.dim())(*t.shape)
            h = L.clove_tensor_create_nd(t.data_ptr(), shp, t.dim(), dt, local)
            if not h:
                raise RuntimeError(_lib.last_error())
            return h

        kv_shape = (C.c_int64 * 5)(*case.pool.storage.shape)
        kv_h = L.clove_tensor_from_device(case.pool.storage.data_ptr(), kv_shape, 5, code, local)
        hq2, hk2, hv2 = hq.view(lay.batch, -1), hk.view(lay.batch, -1), hv.view(lay.batch, -1)

        def e2e_step():
            hs = [mk(hq2, code), mk(hk2, code), mk(hv2, code), mk(hbt, 32), mk(hcl, 32)]
            o = L.clove_paged_attention(hs[0], hs[1], hs[2], kv_h, hs[3], hs[4])
            if not o:
                raise RuntimeError(_lib.last_error())
            L.clove_tensor_data(o, hout.data_ptr())
            for h in hs + [o]:
                L.clove_tensor_free(h)

    for _ in range(3):
        e2e_step()
    _barrier(ws)
    torch.cuda.synchronize()
    e2e_stream = stream if case.head_split else torch.cuda.default_stream(dev)  # the FFI runs on the legacy stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(e2e_stream)
    for _ in range(args.steps):
        e2e_step()
    ev1.record(e2e_stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(ev0.elapsed_time(ev1) / args.steps, ws, dev)
    if not case.head_split:
        kv_h and _lib.lib().clove_tensor_free(kv_h)
    head = config_record(case, ms_max, peak, per_step)
    del hq, hk, hv, hbt, hcl, hout, dq, dk, dv, dbt, dcl
    case.close()
    del case
    gc.collect()
    torch.cuda.empty_cache()

    # ---- the other configurations at the same N, measured in the same run ----
    per_config = {}
    if args.per_config and args.batch is None:
        for name in [c for c in ("c2", "c3", "c4", "c5") if c != args.config]:
            c = DecodeCase(name, ws, rank, dev, weak=args.weak)
            _, cmax, cper, _ = time_case(c, args.steps, args.warmup, local=local)
            rec = config_record(c, cmax, peak, cper)
            rec["phases"] = phase_breakdown(c)
            per_config[name] = rec
            c.close()
            del c
            gc.collect()
            torch.cuda.empty_cache()

    if rank != 0:
        return
    cb = None
    if args.cpu_seconds > 0 and ws == 1:
        lay_s, sample = host_sample_case(spec, args.cpu_seqs)
        cb = cpu_arm(lay_s, sample, args.cpu_seconds)
    achieved = head["hbm_gbs"]
    traffic = args.traffic if args.traffic is not None else (
        None if (args.batch is not None or ws > 1) else TRAFFIC_MEASURED.get(spec.name))
    line = {
        "metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "weak" if head["partition"].endswith("replicas") else "strong",
        "vs_baseline": None, "dtype": _dtype_name(spec.dtype), "data": "synthetic",
        "config": headline_config(args.config, ws, args.weak, args.batch),
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "note": (f"achieved = KV bytes per GPU per step / step time of the slowest rank (plan + "
                              f"decode + combine), peak {peak_kind}; traffic = DRAM bytes per decode launch "
                              f"from an earlier full-size ncu capture of this workload (not this run)"
                              if traffic is not None else
                              f"achieved = KV bytes per GPU per step / step time of the slowest rank, "
                              f"peak {peak_kind}; no ncu capture of this exact case")},
        "phases": breakdown,
        "gpu_launches": launches,
        "clocks": clocks,
        "e2e": {"value": head["global_batch"] / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "cpu_baseline": cb,
        "per_config": per_config,
    }
    print(json.dumps(line), flush=True)


def run_qkv(args) -> None:
    """`--op qkv_append`: the fused Q/K/V projection + KV append
    (clove_cuda_qkv_append) on one GPU, shaped like config C3's decode step
    (hidden 4096 = 32 x 128, 32 q / 8 kv heads, bf16, batch 128 unless
    --batch; --hidden H gives H/128 q heads).  Four packed weight copies rotate (201 MB > L2), so each step
    streams its weights from HBM.  Reports the kernel's weight-streaming
    bandwidth against the measured HBM peak, and the same step done as a
    cuBLAS GEMM + the append kernel for comparison."""
    import torch

    from clove_b200 import KVPool, launch_count
    ws, rank, local = _dist()
    if rank != 0:
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hidden = args.hidden or 4096
    hq, hkv, D, bs = hidden // 128, 8, 128, 16
    B = args.batch or 128
    n_out = (hq + 2 * hkv) * D
    g = torch.Generator(device=dev)
    g.manual_seed(303)
    pool = KVPool(B * 4 + 8, bs, hkv, D, torch.bfloat16, dev)
    x = torch.randn((B, hidden), device=dev, generator=g).bfloat16()
    raw = [(torch.randn((n_out, hidden), device=dev, generator=g) / 64).bfloat16() for _ in range(4)]
    packed = [pool.pack_qkv_weights(w) for w in raw]
    bias = torch.randn(n_out, device=dev, generator=g) * 0.1
    bt = torch.arange(B * 4, device=dev, dtype=torch.int32).reshape(B, 4)
    ctx = torch.randint(0, 4 * bs, (B,), device=dev, dtype=torch.int32, generator=g)
    q = torch.empty((B, hq, D), dtype=torch.bfloat16, device=dev)
    lens = torch.empty(B, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    def graph_of(fns, reps):
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for f in fns:
                f()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(reps):
                fns[i % len(fns)]()
        return gr

    def timed(gr, reps):
        for _ in range(max(args.warmup, 3)):
            gr.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        for _ in range(args.steps):
            gr.replay()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / (args.steps * reps)  # ms per step

    REPS = 20
    fused = [lambda w=w: pool.qkv_append(x, w, bias, hq, bt, ctx, q_out=q, lens_out=lens) for w in packed]
    gr = graph_of(fused, REPS)
    n0 = launch_count()
    fused[0]()  # launches per step, counted on one eager call (graph replays bypass the host)
    per_step = launch_count() - n0
    with ClockSampler(local) as clk:
        ms = timed(gr, REPS)
    launches = per_step * args.steps * REPS
    assert pool.pool_status() == 0
    # library comparison: one cuBLAS GEMM (bias folded in) + the append kernel
    y = torch.empty((B, n_out), dtype=torch.bfloat16, device=dev)
    slots = (bt[torch.arange(B, device=dev), (ctx // bs).long()] * bs + ctx % bs).to(torch.int32)
    bb = bias.bfloat16()

    def lib_step(w):
        torch.addmm(bb, x, w.t(), out=y)
        pool.reshape_and_cache(y[:, hq * D:(hq + hkv) * D].contiguous(), y[:, (hq + hkv) * D:].contiguous(), slots)

    ms_lib = timed(graph_of([lambda w=w: lib_step(w) for w in raw], REPS), REPS)
    # end to end: x from pinned host memory, q back to the host, every step
    xh = x.cpu().pin_memory()
    qh = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    for _ in range(3):
        x.copy_(xh, non_blocking=True)
        pool.qkv_append(x, packed[0], bias, hq, bt, ctx, q_out=q, lens_out=lens)
        qh.copy_(q, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    steps_e2e = min(args.steps, 200)
    a.record()
    for i in range(steps_e2e):
        x.copy_(xh, non_blocking=True)
        pool.qkv_append(x, packed[i % 4], bias, hq, bt, ctx, q_out=q, lens_out=lens)
        qh.copy_(q, non_blocking=True)
    b.record()
    b.synchronize()
    ms_e2e = a.elapsed_time(b) / steps_e2e
    w_bytes = packed[0].numel()
    alg = w_bytes + x.numel() * 2 + n_out * 4 + B * n_out * 2 + B * 4 * 3  # weights, x, bias, q/k/v out, tables
    peak, kind = _peaks()
    achieved = alg / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "fused_qkv_append_tokens_per_s", "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"C3-shaped decode projection: x [{B}, {hidden}] -> q/k/v {hq}q/{hkv}kv x {D}, "
                               f"bf16, K/V into paged slots (bs {bs})",
                   "l2": "4 weight copies rotated (201 MB > L2)", "graph": True},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": kind},
        "library_step_ms": ms_lib, "library_step": "torch.addmm (cuBLAS) + clove reshape_and_cache",
        "e2e": {"value": B / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": q.numel() * 2},
        "gpu_launches": launches, "clocks": clk.summary(),
    }))


def run_prefill(args) -> None:
    """`--op prefill`: causal prefill into the paged cache (clove_cuda_paged_prefill:
    RoPE + cache write + attention) on one GPU, bf16, 32 query / 8 KV heads x
    128, block 32, fresh prompts: `--batch` prompts of `--prompt` tokens
    (default 8 x 2048).  FLOPs per step = batch * Hq * 2 * T^2 * D (QK^T and
    P.V over the causal half).  Reports TFLOP/s against the measured bf16
    tensor peak, and the warp-MMA kernel's time for comparison."""
    import torch

    from clove_b200 import KVPool, launch_count, set_decode_variant
    ws, rank, local = _dist()
    if rank != 0:
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hq, hkv, D, bs = 32, 8, 128, 32
    B, T = (args.batch or 8), args.prompt
    need = (T + bs - 1) // bs
    nb = B * need
    g = torch.Generator(device=dev)
    g.manual_seed(606)
    pool = KVPool(nb, bs, hkv, D, torch.bfloat16, dev)
    pool.storage.normal_(generator=g)
    bt = torch.arange(nb, dtype=torch.int32, device=dev).reshape(B, need)
    cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=dev)
    ctx = torch.zeros(B, dtype=torch.int32, device=dev)
    q = torch.randn((B * T, hq, D), device=dev, generator=g).bfloat16()
    k = torch.randn((B * T, hkv, D), device=dev, generator=g).bfloat16()
    v = torch.randn((B * T, hkv, D), device=dev, generator=g).bfloat16()
    flops = B * hq * 2.0 * T * T * D

    def step():
        return pool.prefill(q, k, v, cu, bt, ctx, max_ctx=T, rope_theta=10000.0)

    def timed(n):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / n

    n0 = launch_count()
    step()
    torch.cuda.synchronize()
    per_step = launch_count() - n0
    with ClockSampler(local) as clk:
        ms = timed(args.steps)
    set_decode_variant("mma")
    try:
        ms_mma = timed(max(3, args.steps // 4))
    finally:
        set_decode_variant("auto")
    assert pool.pool_status() == 0
    # end to end: prompts from pinned host memory, outputs back to host
    hq_, hk_, hv_ = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    out_h = torch.empty((B * T, hq, D), dtype=torch.float32).pin_memory()
    for _ in range(2):
        q.copy_(hq_, non_blocking=True), k.copy_(hk_, non_blocking=True), v.copy_(hv_, non_blocking=True)
        out_h.copy_(step(), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ne = max(3, args.steps // 4)
    e0.record()
    for _ in range(ne):
        q.copy_(hq_, non_blocking=True), k.copy_(hk_, non_blocking=True), v.copy_(hv_, non_blocking=True)
        out_h.copy_(step(), non_blocking=True)
    e1.record()
    e1.synchronize()
    ms_e2e = e0.elapsed_time(e1) / ne
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak, kind = (pk["bf16_tflops"], "measured burst") if "bf16_tflops" in pk else (1590.0, "fallback")
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "paged prefill TFLOP/s (causal)", "value": tf, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"prefill {B} x {T} tokens, 32q/8kv x 128, block 32, RoPE, fresh prompts",
                   "l2": "K/V re-read from L2 by design (causal tiles)"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                     "traffic": None, "peak_kind": kind,
                     "note": "whole call (RoPE + cache write + plan + attention) over the causal FLOPs"},
        "warp_mma_ms_per_step": ms_mma, "warp_mma_tflops": flops / (ms_mma * 1e-3) / 1e12,
        "e2e": {"value": flops / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": (q.numel() + k.numel() + v.numel()) * 2, "d2h_bytes_per_step": out_h.numel() * 4},
        "gpu_launches": per_step * args.steps, "clocks": clk.summary(),
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--op", default="decode", choices=["decode", "qkv_append", "prefill"],
                    help="decode (the headline path), the fused Q/K/V projection + append, or prefill")
    ap.add_argument("--prompt", type=int, default=2048, help="--op prefill: tokens per prompt")
    ap.add_argument("--hidden", type=int, default=None, help="--op qkv_append: model width (default 4096)")
    ap.add_argument("--cpu-seqs", type=int, default=8)
    ap.add_argument("--batch", type=int, default=None, help="override the config batch (profiling only)")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of a captured CUDA graph")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--weak", action="store_true",
                    help="N>1: every rank runs a full replica of the workload instead of a shard of it")
    ap.add_argument("--no-per-config", dest="per_config", action="store_false",
                    help="skip the c2-c5 records measured after the headline")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per decode launch from an ncu capture (reported as roofline.traffic)")
    args = ap.parse_args()
    if args.op == "qkv_append":
        run_qkv(args)
    elif args.op == "prefill":
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
    try:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
