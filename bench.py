"""Benchmark of the MoE-FFN hot path on B200.

Workload (default, --workload resident): gpt-oss-120b-shaped MoE FFN stack,
36 layers, 128 experts per layer with gate_up [5760 x 2880] and down
[2880 x 2880] in MXFP4 (quantized on the device from N(0, 0.02)), top-4
softmax routing over N(0, 1) logits (uniform expert popularity), a 64-token
decode batch with bf16 activations. All experts are resident: with N GPUs
each GPU holds 128/N experts of every layer and 64/N of the tokens, and the
(token, expert) rows are dispatched to the experts' GPUs and the results
combined back with NCCL all-to-all (expert parallelism; total work fixed, so
scaling is strong). One step = the 36 layers for one batch:
remap + grouping -> fused gate/up mul_mat_id + SwiGLU -> down mul_mat_id ->
router-weighted combine (plus dispatch / combine exchanges when N > 1).

The 60.9 GB of expert weights are far larger than L2 (126 MB), so no step
finds its weights in cache.

`value` is tokens/s with inputs resident in HBM; `e2e` is the same step
through the public API with host buffers: the step's activations and routing
copied from pinned host memory and every layer's output read back, inside
the timed region. `--impl reference` times the CPU restatement of the same
path (the oracle's vectorized form of ggml's q8_0 mul_mat_id) on all host
threads, every layer of every step.

`--workload streamed` (1 GPU, not the default line) times the decode with a
slot cache per layer and misses filled from pinned host memory, with the
cache decisions on the device (`--remap device`) or on the host with a round
trip per layer (`--remap host`); see streamed_main. `--workload slots`
(1 GPU) times small decode batches over slot pools whose routed experts are
all resident (`--model gpt-oss` or `iq4nl-256e`); see slots_main.
"""
import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-FFN tokens/s + mul_mat_id HBM GB/s & FP4 TC util at 1/2/4/8 B200"

SHAPE = dict(n_layer=36, n_expert=128, hidden=2880, n_ff=2880, top_k=4, tokens=64)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="msb", choices=["msb", "reference"])
    ap.add_argument("--tokens", type=int, default=SHAPE["tokens"])
    ap.add_argument("--layers", type=int, default=SHAPE["n_layer"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--transport", default="peers", choices=["peers", "collective"],
                    help="expert-parallel exchange: NVLink peer-memory kernels or NCCL all-to-all")
    ap.add_argument("--eager", action="store_true",
                    help="launch every kernel from the host instead of replaying CUDA graphs")
    ap.add_argument("--workload", default="resident",
                    choices=["resident", "streamed", "slots", "prefill", "single-op"],
                    help="resident: every expert in HBM (the default line); streamed: a slot "
                         "cache per layer with misses filled from pinned host memory (1 GPU); "
                         "slots: small decode batches over slot pools (1 GPU, --model); "
                         "prefill: 512-token Zipf prompt batches with ~30%% of each layer's "
                         "experts filled from pinned host memory during the grouped GEMM "
                         "(1 GPU); single-op: one IQ4_NL mul_mat_id over a 32-slot pool behind "
                         "the slot streamer (1 GPU)")
    ap.add_argument("--passes", default="auto", choices=["auto", "narrow", "wide"],
                    help="tensor-core passes per weight tile: by batch size (8 or 24 pairs), "
                         "always 8, or always 24 (MSB_OPT_WIDE_PASSES)")
    ap.add_argument("--iq4nl", default="auto", choices=["auto", "cuda", "tc"],
                    help="IQ4_NL arithmetic: tensor cores for prompt-sized batches (auto), the "
                         "CUDA-core q8_0 form, or the tensor cores wherever shapes allow "
                         "(MSB_OPT_IQ4NL_PATH)")
    ap.add_argument("--miss-frac", type=float, default=0.3,
                    help="prefill: fraction of each layer's referenced experts not resident")
    ap.add_argument("--model", default="gpt-oss", choices=["gpt-oss", "iq4nl-256e"],
                    help="slots: gpt-oss layers (MXFP4, 32 of 128 experts, top-4) or a "
                         "256-expert IQ4_NL model (hidden 2048, expert FFN 512, 64 slots, top-8)")
    ap.add_argument("--slots", type=int, default=32, help="streamed: slots per layer")
    ap.add_argument("--remap", default="device", choices=["device", "host"],
                    help="streamed: cache decisions on the device (one CUDA graph per step) or "
                         "on the host with a round trip per layer")
    args = ap.parse_args()
    if args.workload in ("streamed", "slots") and "--tokens" not in sys.argv:
        args.tokens = 1
    if args.workload == "prefill":
        if "--tokens" not in sys.argv:
            args.tokens = 512
        if "--layers" not in sys.argv:
            args.layers = 4
    if args.workload == "slots" and args.model == "iq4nl-256e" and "--layers" not in sys.argv:
        args.layers = 40
    return args


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    """Samples SM clock, power and clock-event reasons of one GPU every 10 ms
    from a thread (NVML reads only; nothing is changed). Falls back to
    nvidia-smi when NVML cannot be loaded."""
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device):
        import threading
        self.device = device
        self.rows = []
        self.stop_ev = threading.Event()
        self.thread = None
        self.err = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.device)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def _run(self, nv, h):
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((sm, pw, [n for n, b in zip(self.REASONS, bits) if rs & b]))
            except Exception as e:  # keep the bench running; report why
                self.err = str(e)
                return
            self.stop_ev.wait(0.01)

    def start(self):
        import threading
        try:
            nv, h = self._handle()
            self.max_sm = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception as e:
            self.err = f"NVML unavailable: {e}"
            return
        self.thread = threading.Thread(target=self._run, args=(nv, h), daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no sampler"]}
        self.stop_ev.set()
        self.thread.join(timeout=5)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        sm = sorted(r[0] for r in self.rows)
        reasons = sorted({n for r in self.rows for n in r[2]})
        return {"sm_mhz": float(sm[len(sm) // 2]), "sm_max_mhz": float(self.max_sm),
                "reasons": reasons, "samples": len(self.rows),
                "power_w_max": round(max(r[1] for r in self.rows), 1)}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif args.impl == "msb":
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------
def make_routing(g, n_steps, n_layer, tokens, n_expert, top_k):
    """Per (step, layer): top-k ids of N(0,1) logits and softmax weights over the
    selected logits."""
    import torch
    logits = torch.randn(n_steps, n_layer, tokens, n_expert, generator=g, device="cuda")
    sel, ids = torch.topk(logits, top_k, dim=-1)
    w = torch.softmax(sel, dim=-1).float().contiguous()
    return ids.to(torch.int32).contiguous(), w


def build_layers(n_layer, e_lo, e_hi, K, n_ff, seed):
    """Pools (gate, up, down) of this rank's experts [e_lo, e_hi) for every
    layer, quantized on the device from N(0, 0.02). Slot j holds expert
    e_lo + j. The gate_up projection [5760 x 2880] is held as its two halves,
    gate [2880 x 2880] and up [2880 x 2880], so each starts on a 128-row
    boundary for the tensor cores."""
    import torch

    from moestream_b200 import ops
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    n_loc = e_hi - e_lo
    layers = []
    for layer in range(n_layer):
        ga = ops.SlotPool("mxfp4", K, n_ff, n_loc, max_fill_batch=8)
        up = ops.SlotPool("mxfp4", K, n_ff, n_loc, max_fill_batch=8)
        dn = ops.SlotPool("mxfp4", n_ff, K, n_loc, max_fill_batch=8)
        for pool, rows, cols in ((ga, n_ff, K), (up, n_ff, K), (dn, K, n_ff)):
            for j0 in range(0, n_loc, 8):
                j1 = min(n_loc, j0 + 8)
                wts = torch.randn((j1 - j0) * rows, cols, generator=g, device="cuda") * 0.02
                q = ops.quantize_rows("mxfp4", wts).view(j1 - j0, -1)
                pool.fill(list(range(j0, j1)), [q[i] for i in range(j1 - j0)])
                del wts
        layers.append((ga, up, dn))
    torch.cuda.synchronize()
    return layers


def run_layer(ctx, layer, x, ids, w, y, timed_events=None):
    """One MoE FFN layer on this rank. x: [t_loc, K] bf16, ids/w: [t_loc, top_k]."""
    from moestream_b200 import ops
    top_k = ids.shape[1]
    ga, up, dn = ctx["layers"][layer]
    lib = ops.lib()
    if timed_events is not None:
        lib.msb_time_next_gate_up(ops.c_vp(timed_events[0].cuda_event),
                                  ops.c_vp(timed_events[1].cuda_event))
    if ctx["world"] == 1:
        r = ops.remap_group(ids, ga.n_slot, route=ctx["route"])
        ops.moe_ffn(ga, up, dn, x, r, w, top_k, ws=ctx["ws"], out=y)
        return
    ep = ctx["ep"]

    def local_ffn(rows, local_ids, route, out):
        ops.moe_ffn(ga, up, dn, rows, route, None, 1, ws=ctx["ws"], out=out)

    ep.layer(x, ids, w, local_ffn, y, pools=(ga, up, dn, 0, ctx["ws"]))


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(layer0, top_k, K, n_ff, n_expert, ids_step, w_step, x0, threads):
    """Times the CPU baseline (the oracle's vectorized q8 restatement of
    ggml's CPU path, all host threads) on one whole step: every layer's
    routing of the step, each layer over layer 0's weights as read back from
    the GPU's pools (the bytes the GPU read; 1.7 GB, far larger than the host
    caches). Returns seconds per step (best of 2)."""
    import numpy as np

    from oracle import oracle as O
    ga, up, dn = layer0
    gu_h = np.stack([np.concatenate([ga.read_slot(s).cpu().numpy(), up.read_slot(s).cpu().numpy()])
                     for s in range(n_expert)] + [np.zeros(2 * ga.expert_bytes, np.uint8)])
    dn_h = np.stack([dn.read_slot(s).cpu().numpy() for s in range(n_expert)] +
                    [np.zeros(dn.expert_bytes, np.uint8)])
    best = None
    for _ in range(2):
        t0 = time.perf_counter()
        for il in range(ids_step.shape[0]):
            O.moe_ffn_fast("mxfp4", gu_h, gu_h, dn_h, K, n_ff, x0, ids_step[il], w_step[il],
                           up_row0=n_ff, nthreads=threads)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best


# ---------------------------------------------------------------------------
# Reference arm: the CPU restatement on the host cores
# ---------------------------------------------------------------------------
def reference_weight_sets(n_sets, n_base, K, n_ff, E, threads, seed=0):
    """n_sets distinct slot slabs of one layer (fused gate_up [E + 1, 2 x 2880
    rows] and down [E + 1, 2880 rows], ggml MXFP4 bytes, slot E the zero
    slot). Every slot holds its own copy of one of n_base experts per role
    quantized from N(0, 0.02) by the oracle's quantizer (gguf's MXFP4
    algorithm, the same as the GPU arm's device quantizer)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    w_gu = rng.normal(0.0, 0.02, size=(n_base * 2 * n_ff, K)).astype(np.float32)
    w_dn = rng.normal(0.0, 0.02, size=(n_base * K, n_ff)).astype(np.float32)

    def q(a):   # quantize row chunks in parallel (the C call releases the GIL)
        parts = np.array_split(a, threads * 4)
        with ThreadPoolExecutor(threads) as ex:
            return np.concatenate(list(ex.map(lambda c: O.quantize("mxfp4", c), parts)))
    base_gu = q(w_gu).reshape(n_base, -1)
    base_dn = q(w_dn).reshape(n_base, -1)
    del w_gu, w_dn
    sets = []
    for s in range(n_sets):
        gu = np.empty((E + 1, base_gu.shape[1]), np.uint8)
        dn = np.empty((E + 1, base_dn.shape[1]), np.uint8)
        for e in range(E):
            b = (7 * e + 3 * s) % n_base
            gu[e] = base_gu[b]
            dn[e] = base_dn[b]
        gu[E] = 0
        dn[E] = 0
        sets.append((gu, dn))
    return sets


def reference_arm(args, world, rank):
    """The reference's CPU implementation of this path is ggml's CPU
    mul_mat_id (q8_0 activations, int8 block dots), which is not vendored;
    its published algorithm is restated by the oracle (msb_cpu_fast.c,
    vectorized like ggml's x86 code) and timed here on all host threads over
    the whole step: every one of the 36 layers, each with its own routing."""
    if rank != 0:
        return 0
    import numpy as np

    from oracle import oracle as O
    K, n_ff, E, top_k = SHAPE["hidden"], SHAPE["n_ff"], SHAPE["n_expert"], SHAPE["top_k"]
    T, L = args.tokens, args.layers
    threads = host_threads()
    t_setup = time.time()
    # Layer l reads weight set l % n_sets: each set (1.7 GB) is far larger
    # than the host caches, so no layer finds its weights cached, while the
    # host holds 4 sets instead of 36.
    n_sets, n_base = min(L, 4), 4
    sets = reference_weight_sets(n_sets, n_base, K, n_ff, E, threads)
    rng = np.random.default_rng(1)
    S = args.warmup + args.steps
    logits = rng.normal(0, 1, size=(S, L, T, E))
    ids = np.argsort(-logits, axis=-1, kind="stable")[..., :top_k].astype(np.int32)
    sel = np.take_along_axis(logits, ids, -1)
    w = np.exp(sel - sel.max(-1, keepdims=True))
    w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
    del logits, sel
    # bf16-valued activations, as the GPU arm's
    x = rng.normal(0, 1, size=(S, T, K)).astype(np.float32)
    x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)
    t_setup = time.time() - t_setup
    times = []
    for step in range(S):
        t0 = time.perf_counter()
        for il in range(L):
            gu, dn = sets[il % n_sets]
            O.moe_ffn_fast("mxfp4", gu, gu, dn, K, n_ff, x[step], ids[step, il], w[step, il],
                           up_row0=n_ff, nthreads=threads)
        dt = time.perf_counter() - t0
        if step >= args.warmup:
            times.append(dt)
    step_s = sum(times) / len(times)
    v = T / step_s
    macs = 3 * n_ff * K * T * top_k * L
    sample = (f"every step whole: {L} layers x {T} tokens x top-{top_k} ({macs / 1e9:.0f} GMAC); "
              f"{threads} threads, {O.fast_isa()} int8 dots; weights: {n_sets} sets of 128 "
              f"MXFP4 experts from N(0,0.02), layer l reads set l % {n_sets}; CPU "
              "restatement of ggml's q8_0 mul_mat_id (ggml is not available offline)")
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "mxfp4 x q8_0 (int8 dots) -> f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "gpt-oss-120b-shaped MoE FFN decode, all experts resident",
                       "n_layer": L, "n_expert": E, "hidden": K, "n_ff": n_ff,
                       "top_k": top_k, "tokens": T},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "nproc": os.cpu_count(), "isa": O.fast_isa(),
                             "gmac_per_s_per_core": macs / step_s / threads / 1e9,
                             "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "setup_s": round(t_setup, 1)}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Main arm
# ---------------------------------------------------------------------------
def streamed_main(args):
    """--workload streamed: the same gpt-oss-shaped 36-layer decode, but each
    layer keeps only `--slots` experts per role in HBM (a slot cache per
    layer, the reference's decode setting) and every miss is filled from
    pinned host memory while the step runs. Routing adds a per-layer Zipf 1.1
    popularity bias to the N(0, 1) logits, so the caches see locality. The
    experts of one layer are quantized on the device from N(0, 0.02) and kept
    as one pinned host copy per role that every layer's misses read (the
    bytes do not change the timing; pinned memory stays at 1.7 GB).
    --remap device: cache decisions, fills (one launch for the three roles),
    grouping and FFN of all layers in one CUDA graph per step, no host round
    trip; --remap host: each
    layer's ids go to the host, the host slot streamer decides, DMA fills,
    the slots come back. Both make the same decisions."""
    import numpy as np
    import torch

    from moestream_b200 import DeviceSlotStreamer, SlotStreamer, ops
    K, n_ff, E, top_k = SHAPE["hidden"], SHAPE["n_ff"], SHAPE["n_expert"], SHAPE["top_k"]
    T, L, NS = args.tokens, args.layers, args.slots
    t_setup = time.time()
    g = torch.Generator(device="cuda")
    g.manual_seed(4321)
    src = {}
    for role, rows, cols in (("gate", n_ff, K), ("up", n_ff, K), ("down", K, n_ff)):
        parts = []
        for j0 in range(0, E, 8):
            wts = torch.randn(8 * rows, cols, generator=g, device="cuda") * 0.02
            parts.append(ops.quantize_rows("mxfp4", wts).view(8, -1).cpu())
        src[role] = torch.cat(parts).pin_memory()
    pools = [{r: ops.SlotPool("mxfp4", kk, nn, NS, max_fill_batch=8)
              for r, kk, nn in (("gate", K, n_ff), ("up", K, n_ff), ("down", n_ff, K))}
             for _ in range(L)]
    S = args.warmup + args.steps
    ranks = torch.stack([torch.randperm(E, generator=g, device="cuda") for _ in range(L)]) + 1
    bias = torch.log(ranks.double() ** -1.1 / (ranks.double() ** -1.1).sum(1, keepdim=True))
    logits = torch.randn(S, L, T, E, generator=g, device="cuda") + bias.float()[None, :, None]
    sel, ids_all = torch.topk(logits, top_k, dim=-1)
    ids_all = ids_all.to(torch.int32).contiguous()
    w_all = torch.softmax(sel, dim=-1).float().contiguous()
    xs = torch.randn(S, T, K, generator=g, device="cuda").to(torch.bfloat16)
    eb = {r: pools[0][r].expert_bytes for r in src}
    per_expert = sum(eb.values())
    route = ops.RouteBuffers(T * top_k, NS)
    ws = ops.workspace(K, T, top_k, NS)
    y = torch.empty(L, T, K, dtype=torch.float32, device="cuda")
    x_d = torch.empty(T, K, dtype=torch.bfloat16, device="cuda")
    ids_d = torch.empty(L, T, top_k, dtype=torch.int32, device="cuda")
    w_d = torch.empty(L, T, top_k, dtype=torch.float32, device="cuda")
    slots = torch.empty(L, T, top_k, dtype=torch.int32, device="cuda")
    lib = ops.lib()
    # Host-to-device copy bandwidth of this GPU (the fills' bound), measured here.
    big = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    big_d = torch.empty_like(big, device="cuda")
    best = None
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        big_d.copy_(big, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = a.elapsed_time(b) if best is None else min(best, a.elapsed_time(b))
    h2d_gbs = big.numel() / (best / 1e3) / 1e9
    del big, big_d

    def set_inputs(s):
        x_d.copy_(xs[s])
        ids_d.copy_(ids_all[s])
        w_d.copy_(w_all[s])

    roles = ("gate", "up", "down")
    if args.remap == "device":
        dev = DeviceSlotStreamer(L, E, NS, T * top_k, per_expert)

        def step():
            for il in range(L):
                dev.remap(il, ids_d[il], out=slots[il])
                dev.fill_roles(il, [pools[il][r] for r in roles], [src[r] for r in roles])
                ops.remap_group(slots[il], NS, route=route)
                ops.moe_ffn(pools[il]["gate"], pools[il]["up"], pools[il]["down"], x_d, route,
                            w_d[il], top_k, ws=ws, out=y[il])

        def misses():
            return dev.stats()["miss"]
    else:
        host = SlotStreamer(L, E, NS, per_expert)
        n_miss = [0]

        def step():
            for il in range(L):
                ids_h = ids_d[il].cpu().numpy()   # the round trip: waits for the device
                sl, miss, _ = host.remap(il, ids_h)
                if miss:
                    es, ss = [e for e, _ in miss], [q for _, q in miss]
                    for r in ("gate", "up", "down"):
                        pools[il][r].fill(ss, [src[r][e] for e in es])
                    n_miss[0] += len(miss)
                slots[il].copy_(torch.from_numpy(sl), non_blocking=True)
                ops.remap_group(slots[il], NS, route=route)
                ops.moe_ffn(pools[il]["gate"], pools[il]["up"], pools[il]["down"], x_d, route,
                            w_d[il], top_k, ws=ws, out=y[il])

        def misses():
            return n_miss[0]
    for s in range(args.warmup):
        set_inputs(s)
        step()
    torch.cuda.synchronize()
    graph = None
    launches0 = int(lib.msb_kernel_launches())
    if args.remap == "device":
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        launches = (int(lib.msb_kernel_launches()) - launches0) * args.steps
    t_setup = time.time() - t_setup
    m0 = misses()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    time.sleep(0.05)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for i in range(args.steps):
        set_inputs(args.warmup + i)
        if graph is not None:
            graph.replay()
        else:
            step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if graph is None:
        launches = int(lib.msb_kernel_launches()) - launches0
    ms = t0.elapsed_time(t1)
    miss_step = (misses() - m0) / args.steps
    fill_gbs = miss_step * per_expert / (ms / args.steps / 1e3) / 1e9
    line = {"metric": "MoE-FFN decode tokens/s with expert streaming", "impl": "msb",
            "value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "mxfp4 x bf16 as 4 e2m1 terms per 32-block -> f32", "data": "synthetic",
            "config": {"workload": "gpt-oss-120b-shaped MoE FFN decode, slot cache per layer, "
                                   "misses filled from pinned host memory",
                       "n_layer": L, "n_expert": E, "slots_per_layer": NS, "hidden": K,
                       "n_ff": n_ff, "top_k": top_k, "tokens": T,
                       "routing": "top-4 softmax over N(0,1) logits + per-layer Zipf 1.1 bias",
                       "remap": ("device streamer, one CUDA graph per step" if graph is not None
                                 else "host streamer, a round trip per layer"),
                       "l2": "expert bytes far larger than L2"},
            "misses_per_step": miss_step,
            "roofline": {"bound": "pcie", "achieved": fill_gbs, "peak": h2d_gbs, "unit": "GB/s",
                         "frac": fill_gbs / h2d_gbs, "traffic": None,
                         "kernel": "fills (dfill_kernel or DMA + repack)",
                         "peak_source": "pinned host-to-device copy of 1 GiB measured in this run"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clk,
            "setup_s": round(t_setup, 1)}
    print(json.dumps(line), flush=True)
    graph = None
    return 0


def slots_main(args):
    """--workload slots: a decode batch of --tokens tokens through --layers
    MoE layers whose routed experts are all resident in slot pools (the
    reference's decode configurations of a slot cache that hits): gpt-oss
    layers (MXFP4 2880 x 2880 gate, up and down, 32 slots, top-4) or a
    256-expert IQ4_NL model (hidden 2048, expert FFN 512, 64 slots, top-8 plus
    one shared expert).
    Weights quantized on the device from N(0, 0.02); ids are top_k distinct
    random slots per token, new every step and layer. The 256-expert model's
    shared expert is always resident in one more slot of each layer's pools:
    every token's ids end with it, at weight 1 next to the routed experts'
    weights, so it runs in the same grouped matmuls and combine. A batch
    above the slot pool's arena threshold (6 tokens for both models) runs
    over per-layer arenas of every expert instead, routed over all of them,
    as the reference runs it. One CUDA graph per step; the roofline counts
    each distinct referenced slot's bytes once per layer."""
    import torch

    from moestream_b200 import ops
    if args.model == "gpt-oss":
        wtype, K, n_ff, NS, top_k, E = "mxfp4", SHAPE["hidden"], SHAPE["n_ff"], 32, 4, 128
    else:
        wtype, K, n_ff, NS, top_k, E = "iq4_nl", 2048, 512, 64, 8, 256
    T, L = args.tokens, args.layers
    # Batches the slot pool cannot serve (the reference's arena threshold,
    # msb_arena_threshold) run as the reference runs them: over per-layer
    # arenas holding every expert, routed over all of them.
    threshold = int(ops.lib().msb_arena_threshold(E, top_k, NS))
    arena = T > threshold
    if arena:
        NS = E
    # The 256-expert model's shared expert: slot NS of every pool.
    shared = 1 if args.model != "gpt-oss" else 0
    NSP, top_k_all = NS + shared, top_k + shared
    t_setup = time.time()
    g = torch.Generator(device="cuda")
    g.manual_seed(77)

    def qpool(kk, nn):
        pool = ops.SlotPool(wtype, kk, nn, NSP, max_fill_batch=8)
        for j0 in range(0, NSP, 8):
            j1 = min(NSP, j0 + 8)
            wts = torch.randn((j1 - j0) * nn, kk, generator=g, device="cuda") * 0.02
            q = ops.quantize_rows(wtype, wts).view(j1 - j0, -1)
            pool.fill(list(range(j0, j1)), [q[i] for i in range(j1 - j0)])
        return pool
    layers = [(qpool(K, n_ff), qpool(K, n_ff), qpool(n_ff, K)) for _ in range(L)]
    S = args.warmup + args.steps
    ids_all = torch.rand(S, L, T, NS, generator=g, device="cuda").argsort(dim=-1)[..., :top_k]
    if shared:
        ids_all = torch.cat([ids_all, torch.full((S, L, T, 1), NS, device="cuda")], dim=-1)
    ids_all = ids_all.to(torch.int32).contiguous()
    w = torch.full((T, top_k_all), 1.0 / top_k, device="cuda")
    if shared:
        w[:, top_k] = 1.0
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(L, T, K, dtype=torch.float32, device="cuda")
    route = ops.RouteBuffers(T * top_k_all, NSP)
    ws = ops.workspace(max(K, n_ff), T, top_k_all, NSP)
    ids_d = torch.empty(L, T, top_k_all, dtype=torch.int32, device="cuda")
    eb = sum(p.expert_bytes for p in layers[0])
    lib = ops.lib()

    def step():
        for il in range(L):
            r = ops.remap_group(ids_d[il], NSP, route=route)
            ga, up, dn = layers[il]
            ops.moe_ffn(ga, up, dn, x, r, w, top_k_all, ws=ws, out=y[il])
    for s_ in range(args.warmup):
        ids_d.copy_(ids_all[s_])
        step()
    torch.cuda.synchronize()
    c0 = int(lib.msb_kernel_launches())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    launches = (int(lib.msb_kernel_launches()) - c0) * args.steps
    graph.replay()
    torch.cuda.synchronize()
    t_setup = time.time() - t_setup
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    time.sleep(0.05)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for i in range(args.steps):
        ids_d.copy_(ids_all[args.warmup + i])
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    timed = ids_all[args.warmup:].view(args.steps * L, T * top_k_all).cpu()
    distinct = sum(len(torch.unique(row)) for row in timed)
    gbs = distinct * eb / (ms / 1e3) / 1e9
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    line = {"metric": "MoE-FFN decode tokens/s over slot pools", "impl": "msb",
            "value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "us_per_layer": ms * 1e3 / args.steps / L,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("mxfp4 x bf16 as 4 e2m1 terms per 32-block -> f32" if wtype == "mxfp4"
                      else "iq4_nl x q8_0 -> f32 (CUDA cores) or f16 x f16 -> f32 (tensor cores, "
                           "prompt-sized batches)"),
            "data": "synthetic",
            "config": {"workload": (f"{args.model} MoE FFN decode over {NS}-slot pools, every "
                                    "referenced expert resident" if not arena else
                                    f"{args.model} MoE FFN decode of a batch above the slot "
                                    f"pool's threshold ({threshold} tokens): per-layer arenas "
                                    f"of all {E} experts"),
                       "n_layer": L, "slots": NS, "hidden": K, "n_ff": n_ff, "top_k": top_k,
                       "shared_experts": shared,
                       "tokens": T, "distinct_per_layer": distinct / (args.steps * L),
                       "l2": "random slots every step and layer; pools far larger than L2"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / hbm, "traffic": None,
                         "kernel": "whole step (algorithmic expert bytes / step time)",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clk,
            "setup_s": round(t_setup, 1)}
    print(json.dumps(line), flush=True)
    graph = None
    return 0


def prefill_main(args):
    """--workload prefill: prompt processing of --tokens (512) tokens through
    --layers (4) gpt-oss-shaped layers whose pools hold one slot per expert
    (the arena size the reference uses for prompt batches), with Zipf(1.1)
    expert popularity per layer (top-4 softmax over N(0,1) logits plus
    log p_e, p_e ~ rank^-1.1 over a per-layer permutation). At every step
    --miss-frac (30%) of each layer's referenced experts are not resident:
    a side stream fills them from pinned host memory (msb_fill_slots_async:
    one cudaMemcpyAsync per expert and role, then the repack kernel), one
    layer after the other, while the compute stream runs each layer's grouped
    GEMM over its resident experts; the filled experts' pairs follow in a
    second FFN call that waits on the layer's fill event and adds into y.
    Reported: tokens/s of that overlapped step, and from the same run the
    fills alone, the compute alone (every expert resident) and the two one
    after the other; overlap = (serial - overlapped) / min(fills, compute)."""
    import numpy as np
    import torch

    from moestream_b200 import ops
    K, n_ff, E, top_k = SHAPE["hidden"], SHAPE["n_ff"], SHAPE["n_expert"], SHAPE["top_k"]
    T, L = args.tokens, args.layers
    t_setup = time.time()
    # One layer's experts quantized on the device and kept as pinned host
    # copies; every layer's pools start from them and its misses are filled
    # from them.
    (g0, u0, d0), = build_layers(1, 0, E, K, n_ff, seed=4321)
    host = [torch.stack([p.read_slot(e) for e in range(E)]).cpu().pin_memory()
            for p in (g0, u0, d0)]
    for p in (g0, u0, d0):
        p.close()
    del g0, u0, d0
    torch.cuda.synchronize()
    layers = []
    for _ in range(L):
        pools = tuple(ops.SlotPool("mxfp4", kk, nn, E, max_fill_batch=64)
                      for kk, nn in ((K, n_ff), (K, n_ff), (n_ff, K)))
        for p, h in zip(pools, host):
            for j0 in range(0, E, 64):
                p.fill(list(range(j0, min(E, j0 + 64))), [h[e] for e in range(j0, min(E, j0 + 64))])
        layers.append(pools)
    torch.cuda.synchronize()
    S = args.warmup + args.steps
    rng = np.random.default_rng(11)
    ids, w, pending = [], [], []
    for s_ in range(S):
        ids.append([])
        w.append([])
        pending.append([])
        for il in range(L):
            perm_rng = np.random.default_rng(1000 + il)   # the layer's popularity order
            ranks = perm_rng.permutation(E) + 1
            bias = np.log(ranks ** -1.1 / (ranks ** -1.1).sum())
            logits = rng.normal(0, 1, size=(T, E)) + bias
            i_ = np.argsort(-logits, axis=1, kind="stable")[:, :top_k].astype(np.int32)
            sel = np.take_along_axis(logits, i_, 1)
            w_ = np.exp(sel - sel.max(1, keepdims=True))
            ids[-1].append(torch.from_numpy(i_).cuda())
            w[-1].append(torch.from_numpy((w_ / w_.sum(1, keepdims=True)).astype(np.float32)).cuda())
            ref = np.unique(i_)
            n_miss = int(round(args.miss_frac * len(ref)))
            pending[-1].append(np.sort(rng.choice(ref, n_miss, replace=False)).astype(np.int32))
    tables = []
    for s_ in range(S):
        tables.append([])
        for il in range(L):
            ta = np.arange(E, dtype=np.int32)
            ta[pending[s_][il]] = -1
            tb = np.full(E, -1, dtype=np.int32)
            tb[pending[s_][il]] = pending[s_][il]
            tables[-1].append((torch.from_numpy(ta).cuda(), torch.from_numpy(tb).cuda()))
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(L, T, K, dtype=torch.float32, device="cuda")
    ws = ops.workspace(K, T, top_k, E)
    ra, rb = ops.RouteBuffers(T * top_k, E), ops.RouteBuffers(T * top_k, E)
    side = torch.cuda.Stream()
    main_s = torch.cuda.current_stream()
    lib = ops.lib()
    eb = sum(p.expert_bytes for p in layers[0])
    torch.cuda.synchronize()
    t_setup = time.time() - t_setup

    def fills(s_, il, stream):
        for p, h in zip(layers[il], host):
            es = pending[s_][il].tolist()
            p.fill(es, [h[e] for e in es], stream=stream)

    def compute_all_resident(s_, il):
        ga, up, dn = layers[il]
        r = ops.remap_group(ids[s_][il], E, route=ra)
        ops.moe_ffn(ga, up, dn, x, r, w[s_][il], top_k, ws=ws, out=y[il])

    def timed(fn, s_):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(main_s)
        fn(s_)
        b.record(main_s)
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    def step_overlapped(s_):
        start = torch.cuda.Event()
        start.record(main_s)
        side.wait_event(start)
        for il in range(L):
            ga, up, dn = layers[il]
            ta, tb = tables[s_][il]
            r = ops.remap_group(ids[s_][il], E, table=ta, n_expert=E, route=ra)
            ops.moe_ffn(ga, up, dn, x, r, w[s_][il], top_k, ws=ws, out=y[il])
            fills(s_, il, side)
            done = torch.cuda.Event()
            done.record(side)
            main_s.wait_event(done)
            r = ops.remap_group(ids[s_][il], E, table=tb, n_expert=E, route=rb)
            ops.moe_ffn(ga, up, dn, x, r, w[s_][il], top_k, ws=ws, out=y[il], accumulate=True)

    def step_fills(s_):
        for il in range(L):
            fills(s_, il, main_s)

    def step_compute(s_):
        for il in range(L):
            compute_all_resident(s_, il)

    def step_serial(s_):
        step_fills(s_)
        step_compute(s_)

    for s_ in range(args.warmup):
        step_overlapped(s_)
        step_serial(s_)
    torch.cuda.synchronize()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    time.sleep(0.05)
    c0 = int(lib.msb_kernel_launches())
    t_over = [timed(step_overlapped, args.warmup + i) for i in range(args.steps)]
    launches = int(lib.msb_kernel_launches()) - c0
    clk = clocks.stop()
    t_fill = [timed(step_fills, args.warmup + i) for i in range(args.steps)]
    t_comp = [timed(step_compute, args.warmup + i) for i in range(args.steps)]
    t_ser = [timed(step_serial, args.warmup + i) for i in range(args.steps)]
    ms = sum(t_over) / len(t_over)
    ms_fill, ms_comp, ms_ser = (sum(v) / len(v) for v in (t_fill, t_comp, t_ser))
    miss = [len(pending[args.warmup + i][il]) for i in range(args.steps) for il in range(L)]
    distinct = [len(np.unique(ids[args.warmup + i][il].cpu().numpy())) for i in range(args.steps)
                for il in range(L)]
    fill_bytes = sum(miss) / args.steps * eb
    fill_gbs = fill_bytes / (ms_fill / 1e3) / 1e9
    # pinned host-to-device copy bandwidth, the fills' bound, measured here
    big = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    big_d = torch.empty_like(big, device="cuda")
    best = None
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        big_d.copy_(big, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = a.elapsed_time(b) if best is None else min(best, a.elapsed_time(b))
    h2d_gbs = big.numel() / (best / 1e3) / 1e9
    del big, big_d
    comp_bytes = sum(distinct) / args.steps * eb
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    overlap = (ms_ser - ms) / min(ms_fill, ms_comp) if min(ms_fill, ms_comp) > 0 else None
    line = {"metric": "MoE-FFN prefill tokens/s with slot fills overlapped", "impl": "msb",
            "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "mxfp4 x bf16 as 4 e2m1 terms per 32-block -> f32", "data": "synthetic",
            "config": {"workload": "gpt-oss-120b-shaped MoE FFN prefill, one slot per expert, "
                                   f"{args.miss_frac:.0%} of each layer's referenced experts "
                                   "filled from pinned host memory during the step",
                       "n_layer": L, "n_expert": E, "hidden": K, "n_ff": n_ff, "top_k": top_k,
                       "tokens": T, "routing": "top-4 softmax over N(0,1) logits + per-layer "
                                               "Zipf(1.1) bias",
                       "distinct_per_layer": sum(distinct) / len(distinct),
                       "misses_per_layer": sum(miss) / len(miss),
                       "l2": "expert bytes per step far larger than L2"},
            "fills_ms": ms_fill, "compute_ms": ms_comp, "serial_ms": ms_ser,
            "overlap": overlap,
            "fill_gbs": fill_gbs, "pinned_h2d_gbs": h2d_gbs,
            "compute_gbs": comp_bytes / (ms_comp / 1e3) / 1e9,
            "roofline": {"bound": "pcie", "achieved": fill_gbs, "peak": h2d_gbs, "unit": "GB/s",
                         "frac": fill_gbs / h2d_gbs, "traffic": None,
                         "kernel": "fills (cudaMemcpyAsync + repack), side stream",
                         "peak_source": "pinned host-to-device copy of 1 GiB measured in this "
                                        "run",
                         "compute_frac_of_hbm": comp_bytes / (ms_comp / 1e3) / 1e9 / hbm},
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clk,
            "setup_s": round(t_setup, 1)}
    print(json.dumps(line), flush=True)
    return 0


def single_op_main(args):
    """--workload single-op: the single mul_mat_id op -- 128 IQ4_NL experts
    [768 x 2048] quantized from N(0, 0.02), a 32-slot pool warmed with a
    seeded subset, one f32 token per step whose top-8 of N(0, 1) router
    logits go through the slot streamer (host remap, misses filled from
    pinned host memory first, untimed), then the timed part: grouping and
    mul_mat_id on the device. The roofline counts the 8 experts' bytes."""
    import numpy as np
    import torch

    from moestream_b200 import SlotStreamer, ops
    wtype, K, N, E, S_, top_k = "iq4_nl", 2048, 768, 128, 32, 8
    T = args.tokens
    t_setup = time.time()
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    host = []
    for j0 in range(0, E, 16):
        wts = torch.randn(16 * N, K, generator=g, device="cuda") * 0.02
        host.append(ops.quantize_rows(wtype, wts).view(16, -1).cpu())
    host = torch.cat(host).pin_memory()
    pool = ops.SlotPool(wtype, K, N, S_, max_fill_batch=8)
    streamer = SlotStreamer(1, E, S_, pool.expert_bytes)
    rng = np.random.default_rng(1)
    subset = rng.permutation(E)[:S_].astype(np.int32)

    def fill(misses):
        if misses:
            pool.fill([s for _, s in misses], [host[e] for e, _ in misses])
    for c in range(S_ // top_k):
        fill(streamer.remap(0, subset[top_k * c:top_k * (c + 1)].reshape(1, top_k))[1])
    rng = np.random.default_rng(3)
    route = ops.RouteBuffers(T * top_k, S_)
    ws = ops.workspace(K, T, top_k, S_)
    out = torch.empty(T, top_k, N, dtype=torch.float32, device="cuda")
    b = torch.from_numpy(np.random.default_rng(2).normal(0, 1, size=(T, 1, K))
                         .astype(np.float32)).cuda()
    torch.cuda.synchronize()
    t_setup = time.time() - t_setup
    times, misses_n = [], 0
    clocks = Clocks(torch.cuda.current_device())
    # The op (grouping, activation quantization, mul_mat_id) 20 times in one
    # CUDA graph over a device copy of the step's slot ids, so the timing is
    # the device's, not the host's launch rate.
    slots_d = torch.zeros(T, top_k, dtype=torch.int32, device="cuda")

    def op():
        r = ops.remap_group(slots_d, S_, route=route)
        ops.mul_mat_id(pool, b, r, top_k, ws=ws, out=out)
    op()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(20):
            op()
    for step in range(args.warmup + args.steps):
        logits = rng.normal(0, 1, size=(T, E))
        ids = np.argsort(-logits, axis=1, kind="stable")[:, :top_k].astype(np.int32)
        slots, misses, _ = streamer.remap(0, ids)
        fill(misses)
        slots_d.copy_(torch.from_numpy(slots))
        torch.cuda.synchronize()
        if step == args.warmup:
            clocks.start()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        if step >= args.warmup:
            times.append(a.elapsed_time(e) / 20)
            misses_n += len(misses)
    graph = None
    clk = clocks.stop()
    us = sum(times) / len(times) * 1e3
    gbs = len(np.unique(slots)) * pool.expert_bytes / (us / 1e6) / 1e9
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    line = {"metric": "single mul_mat_id op: us per op", "impl": "msb", "value": us,
            "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "iq4_nl x q8_0 -> f32", "data": "synthetic",
            "config": {"workload": "single IQ4_NL mul_mat_id, 128 experts [768 x 2048], 32-slot "
                                   "pool, top-8 through the slot streamer (misses filled before "
                                   "the timed op)", "tokens": T,
                       "misses_per_step": misses_n / args.steps,
                       "timed": "grouping + activation quantization + mul_mat_id, 20 calls "
                                "replayed from one CUDA graph per step"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / hbm, "traffic": None,
                         "kernel": "route + quantize + gemv (the referenced experts' bytes / "
                                   "op time)",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"},
            "cpu_baseline": None, "e2e": None, "gpu_launches": 3 * 20 * args.steps,
            "clocks": clk, "setup_s": round(t_setup, 1)}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "msb" and args.passes != "auto":
        from moestream_b200 import ops
        from moestream_b200._lib import OPT_WIDE_PASSES
        ops.check(ops.lib().msb_set_option(OPT_WIDE_PASSES, {"narrow": 1, "wide": 2}[args.passes]))
    if args.impl == "msb" and args.iq4nl != "auto":
        from moestream_b200 import ops
        from moestream_b200._lib import OPT_IQ4NL_PATH
        ops.check(ops.lib().msb_set_option(OPT_IQ4NL_PATH, {"cuda": 1, "tc": 2}[args.iq4nl]))
    if args.workload == "single-op":
        if args.gpus != 1 or args.impl != "msb":
            print(json.dumps({"workload": "single-op", "unavailable": "one GPU, --impl msb only"}))
            return 0
        if "--tokens" not in sys.argv:
            args.tokens = 1
        return single_op_main(args)
    if args.workload == "prefill":
        if args.gpus != 1 or args.impl != "msb":
            print(json.dumps({"workload": "prefill", "unavailable": "one GPU, --impl msb only"}))
            return 0
        return prefill_main(args)
    if args.workload == "slots":
        if args.gpus != 1 or args.impl != "msb":
            print(json.dumps({"workload": "slots", "unavailable": "one GPU, --impl msb only"}))
            return 0
        return slots_main(args)
    if args.workload == "streamed":
        if args.gpus != 1 or args.impl != "msb":
            print(json.dumps({"workload": "streamed", "unavailable": "one GPU, --impl msb only"}))
            return 0
        return streamed_main(args)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        rc = reference_arm(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc
    import numpy as np
    import torch

    from moestream_b200 import ops
    from moestream_b200.ep import ExpertParallel
    K, n_ff, E, top_k = SHAPE["hidden"], SHAPE["n_ff"], SHAPE["n_expert"], SHAPE["top_k"]
    T, L = args.tokens, args.layers
    assert T % world == 0 and E % world == 0
    n_loc = E // world
    t_loc = T // world
    t_setup = time.time()
    layers = build_layers(L, rank * n_loc, (rank + 1) * n_loc, K, n_ff, seed=1234 + rank)
    S = args.warmup + args.steps
    g = torch.Generator(device="cuda")
    g.manual_seed(99)  # same routing on every rank; each takes its token slice
    ids_all, w_all = make_routing(g, S, L, T, E, top_k)
    xs = (torch.randn(S, T, K, generator=g, device="cuda")).to(torch.bfloat16)
    ids_loc = ids_all[:, :, rank * t_loc:(rank + 1) * t_loc].contiguous()
    w_loc = w_all[:, :, rank * t_loc:(rank + 1) * t_loc].contiguous()
    x_loc = xs[:, rank * t_loc:(rank + 1) * t_loc].contiguous()
    rows_max = T * top_k if world == 1 else world * t_loc * top_k
    ctx = {"layers": layers, "world": world,
           "route": ops.RouteBuffers(rows_max, n_loc),
           "ws": ops.workspace(K, rows_max if world > 1 else T, 1 if world > 1 else top_k, n_loc),
           "ep": (ExpertParallel(world, rank, E, T, top_k, K, "cuda", transport=args.transport)
                  if world > 1 else None)}
    y = torch.empty(L, t_loc, K, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    t_setup = time.time() - t_setup

    def step(x_s, ids_s, w_s, events=None):
        for layer in range(L):
            ev = events[layer] if events is not None else None
            run_layer(ctx, layer, x_s, ids_s[layer], w_s[layer], y[layer], ev)

    lib = ops.lib()

    def capture(fn):
        """CUDA graph of one step (the launches of 36 layers replay without
        host work); returns the graph and the library kernels it holds."""
        graph = torch.cuda.CUDAGraph()
        c0 = int(lib.msb_kernel_launches())
        with torch.cuda.graph(graph):
            fn()
        return graph, int(lib.msb_kernel_launches()) - c0

    for s in range(args.warmup):
        step(x_loc[s], ids_loc[s], w_loc[s])
    torch.cuda.synchronize()
    barrier(world)
    # Dominant kernel timing: events around every fused gate/up launch,
    # recorded by the graphs as external event nodes.
    gate_ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(L)] for _ in range(args.steps)]
    for pair in gate_ev:  # torch creates the CUDA event on its first record
        for a, b in pair:
            a.record()
            b.record()
    torch.cuda.synchronize()
    graphs, launches = [], 0
    if args.eager:
        launches0 = int(lib.msb_kernel_launches())
    else:
        for i in range(args.steps):
            s = args.warmup + i
            g_i, n_i = capture(lambda: step(x_loc[s], ids_loc[s], w_loc[s], gate_ev[i]))
            graphs.append(g_i)
            launches += n_i
        # First replay of each graph uploads it; not timed.
        for g_i in graphs:
            g_i.replay()
    torch.cuda.synchronize()
    from moestream_b200 import ops as _ops
    setup_status = _ops.device_status(clear=True)   # warm-up and graph uploads
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.05)
    def timed_steps():
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        t0.record()
        for i in range(args.steps):
            if args.eager:
                s = args.warmup + i
                step(x_loc[s], ids_loc[s], w_loc[s], gate_ev[i])
            else:
                graphs[i].replay()
        t1.record()
        torch.cuda.synchronize()
        barrier(world)
        # Status bits of the timed steps' kernels: 0 unless a bounded wait
        # gave up (that launch then stalled for the wait limit, one second,
        # and left its results incomplete).
        return t0.elapsed_time(t1), _ops.device_status(clear=True)

    if args.eager:
        launches0 = int(lib.msb_kernel_launches())
    ms, timed_status = timed_steps()
    retry = None
    if max_over_ranks(float(timed_status != 0), world) > 0:
        # A launch of the timed steps failed: the timing is of a broken step.
        # Measure once more and report both attempts.
        print(f"bench: a bounded wait gave up in the timed steps (status {timed_status:#x}); "
              "measuring once more", file=sys.stderr, flush=True)
        retry = {"first_ms_per_step": max_over_ranks(ms, world) / args.steps,
                 "first_status": timed_status}
        ms, timed_status = timed_steps()
    if args.eager:
        launches = (int(lib.msb_kernel_launches()) - launches0) // (2 if retry else 1)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world)
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)

    # Roofline of the fused gate/up mul_mat_id (this rank's launches).
    ids_np = ids_all.cpu().numpy()
    ebytes_gu = 2 * ops.expert_bytes("mxfp4", K, n_ff)  # gate + up
    tot_bytes, tot_ms = 0.0, 0.0
    for i in range(args.steps):
        s = args.warmup + i
        for layer in range(L):
            e = np.unique(ids_np[s, layer].reshape(-1))
            distinct = int(((e >= rank * n_loc) & (e < (rank + 1) * n_loc)).sum())
            # activation terms read (4 x (16 + 4) B per block and pair) and
            # SwiGLU terms written for the down projection
            act = T * top_k * ((K // 32) + (n_ff // 32)) * 4 * 20
            tot_bytes += distinct * ebytes_gu + act
            tot_ms += gate_ev[i][layer][0].elapsed_time(gate_ev[i][layer][1])
    gate_gbs = tot_bytes / (tot_ms / 1e3) / 1e9
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    # DRAM bytes (read + write) of one gate/up launch of this workload: the
    # mean of two launches of a 1-pass ncu capture of the same layer shape
    # (dram__bytes_read.sum + dram__bytes_write.sum; the decode summary under
    # profiles/); other shapes: unmeasured.
    traffic = 0.969e9 if (world == 1 and T == SHAPE["tokens"]) else None
    # Graphs holding NCCL calls must be gone before the process group is
    # destroyed.
    graphs.clear()
    g_i = None

    # End to end with host buffers: every step copies its activations and
    # routing from pinned host memory into the buffers a captured step reads,
    # replays it, and reads every layer's output back to pinned host memory.
    e2e = None
    if not args.no_e2e:
        x_h = x_loc.cpu().pin_memory()
        ids_h = ids_loc.cpu().pin_memory()
        w_h = w_loc.cpu().pin_memory()
        y_h = torch.empty(L, t_loc, K, dtype=torch.float32).pin_memory()
        x_d = torch.empty_like(x_loc[0])
        ids_d = torch.empty_like(ids_loc[0])
        w_d = torch.empty_like(w_loc[0])
        h2d = x_h[0].numel() * 2 + ids_h[0].numel() * 4 + w_h[0].numel() * 4
        d2h = y_h.numel() * 4
        g_e2e = None
        if args.eager:
            run = lambda: step(x_d, ids_d, w_d)
        else:
            g_e2e, _ = capture(lambda: step(x_d, ids_d, w_d))
            run = g_e2e.replay
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        e0.record()
        for i in range(args.steps):
            s = args.warmup + i
            x_d.copy_(x_h[s], non_blocking=True)
            ids_d.copy_(ids_h[s], non_blocking=True)
            w_d.copy_(w_h[s], non_blocking=True)
            run()
            y_h.copy_(y, non_blocking=True)
            torch.cuda.current_stream().synchronize()  # the step's result is on the host
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        e_ms = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {"value": T * args.steps / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}
        run = g_e2e = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O
        threads = host_threads()
        s = args.warmup
        t_step = cpu_sample(layers[0], top_k, K, n_ff, E, ids_np[s], w_all[s].cpu().numpy(),
                            xs[s].float().cpu().numpy(), threads)
        cpu = {"value": T / t_step, "unit": "tokens/s", "cores": threads, "kind": "port",
               "nproc": os.cpu_count(), "isa": O.fast_isa(),
               "sample": f"step {s} whole ({L} layers x {T} tokens, each layer's own routing), "
                         "every layer over layer 0's weights read back from the GPU pools, "
                         "best of 2; CPU restatement of ggml's q8_0 mul_mat_id, vectorized "
                         "(ggml is not available offline)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "mxfp4 x bf16 as 4 e2m1 terms per 32-block -> f32", "data": "synthetic",
                "config": {"workload": "gpt-oss-120b-shaped MoE FFN decode, all experts resident"
                                       + (", expert-parallel" if world > 1 else ""),
                           "n_layer": L, "n_expert": E, "hidden": K, "n_ff": n_ff,
                           "top_k": top_k, "tokens": T, "experts_per_gpu": n_loc,
                           "weights": "MXFP4 from N(0,0.02), quantized on device",
                           "routing": "top-4 softmax over N(0,1) logits",
                           "activations": "bf16 N(0,1)",
                           "l2": "inputs larger than L2 (60.9 GB of expert weights)",
                           "parallelism": f"ep{world}",
                           "exchange": (None if world == 1 else
                                        "NVLink peer-memory kernels" if args.transport == "peers"
                                        else "NCCL all-to-all"),
                           "launch": "eager" if args.eager else "one CUDA graph per step"},
                "roofline": {"bound": "hbm", "achieved": gate_gbs, "peak": hbm, "unit": "GB/s",
                             "frac": gate_gbs / hbm, "traffic": traffic,
                             "kernel": "tc_kernel<2> (fused gate/up mul_mat_id, tcgen05 mxf4)",
                             "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clk,
                "device_status": {"timed": timed_status, "before": setup_status,
                                  "retried": retry},
                "setup_s": round(t_setup, 1)}
        print(json.dumps(line), flush=True)
    if world > 1:
        import gc

        import torch.distributed as dist
        gc.collect()
        torch.cuda.synchronize()
        ctx["ep"].close()
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
