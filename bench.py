"""Decode throughput of a Llama-7B-shape int4 (group-32) stack on B200.

One step = one decode token for every sequence of the batch through all 32
layers plus the int4 lm_head and argmax, with a 2048-entry KV cache
prefilled, run through the plugin ABI (libstrata_b200.so, strata_plugin_v1).
``--model 70b`` runs the 70B-shape stack instead (80 layers, hidden 8192,
64 query / 8 kv heads, FFN 28672, int4 g32) at batch 32 with a 4096-entry KV
cache; its vocabulary is not specified, so that step has no embedding and no
lm_head (hidden states in, hidden states out).

  value  device-timed tokens/s: CUDA events on the plugin's stream around K
         CUDA-graph replays, inputs resident in HBM (max over ranks).
  e2e    the same steps through the ABI with host buffers: each step writes
         the token ids and positions from pinned host memory, runs, and reads
         the next ids back (blocking ABI copies inside the timed region).

N > 1 runs the same model tensor-parallel over N GPUs (q/k/v/gate/up column
shards, o/down row shards, an NCCL all-reduce after o_proj and down_proj):
total work is fixed, so scaling is "strong".

``--impl reference`` times the CPU oracle (a restatement of the reference's
CPU backend plus the decoder ops it lacks) on this host's cores instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ferrite-strata_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from strata_host.blocks import LLAMA_7B, LLAMA_70B, decoder_graph, ffn_shard  # noqa: E402

METRIC = "decode tokens/s, 7B-shape int4 g32 stack"
KV_FILL = 2048            # prefilled cache entries; the new token sits at position 2048
# --model: shape, default batch, prefilled KV entries, metric name
MODELS = {
    "7b": (LLAMA_7B, 8, KV_FILL, METRIC),
    "70b": (LLAMA_70B, 32, 4096, "decode tokens/s, 70B-shape int4 g32 stack (no embedding / lm_head)"),
}
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
# The decode GEMV's sources: a DRAM-traffic figure below is used only while
# these files are unchanged since it was measured.
GEMV_SOURCES = ("ferrite-strata_b200/csrc/k_gemv_mma.cu", "ferrite-strata_b200/csrc/k_int4.cuh")
# DRAM bytes read + written by one launch of the gate/up GEMV with the SwiGLU
# epilogue (ncu: dram__bytes_read.sum + dram__bytes_write.sum of one launch,
# cold cache, in a 2-layer decode step), keyed by (source digest, M, N, K).
GEMV_TRAFFIC = {
    ("c77fdfffe812c0b9", 8, 22016, 4096): 50817792 + 6656,
    ("c77fdfffe812c0b9", 1, 22016, 4096): 50760192 + 11008,
}


def gemv_source_digest():
    import hashlib
    h = hashlib.sha256()
    for rel in GEMV_SOURCES:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def measured_traffic(m, n, k):
    """The measured DRAM traffic of the current GEMV source at this shape, or
    None when it has not been measured."""
    try:
        return GEMV_TRAFFIC.get((gemv_source_digest(), m, n, k))
    except OSError:
        return None


def step_bytes(shape, batch, kv_fill=KV_FILL):
    """Algorithmic HBM bytes of one decode step (whole job): every int4
    weight and bf16 scale once, the KV cache read over kv_fill + 1 positions,
    the new k/v rows written."""
    D, H, G, d, F, V, L = (shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn,
                           shape.vocab, shape.layers)
    mats = [(H * d, D), (G * d, D), (G * d, D), (D, H * d), (F, D), (F, D), (D, F)]
    w = sum(n * k // 2 + n * (k // 32) * 2 for n, k in mats) * L + V * D // 2 + V * (D // 32) * 2
    kv = 2 * batch * G * (kv_fill + 1) * d * 2 * L
    return w + kv


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock, its maximum and the clock-event reasons through NVML
    every 5 ms in a background thread while the timed region runs (reading
    only; no setting is changed)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, reasons))
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._stop:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [m for m, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------
class Model:
    """A decoder stack resident on one GPU (one tensor-parallel shard).  A
    shape without a vocabulary has no embedding and no head: its step input
    is the hidden state and its output the last layer's hidden state."""

    def __init__(self, plugin, torch, batch, rank, world, layers, fmt="w4g32", seq=1, head="argmax",
                 shape=LLAMA_7B, kv_fill=KV_FILL, kv_page=0):
        from strata_host import Device
        self.plugin, self.torch, self.batch, self.seq = plugin, torch, batch, seq
        prefill = seq > 1
        max_len = seq if prefill else kv_fill + 64
        if kv_page:  # a whole number of pages per sequence
            max_len = -(-max_len // kv_page) * kv_page
        self.embed = shape.vocab > 0
        if not self.embed:
            head = "none"
        g, hd = decoder_graph(shape, batch=batch, seq=seq, max_len=max_len, fmt=fmt, layers=layers,
                              embed=self.embed, head=head, tp_rank=rank, tp_world=world, last_token=prefill,
                              kv_page=kv_page)
        self.graph, self.hd = g, hd
        lib = C.CDLL(plugin.path)
        q4 = lib.strata_b200_quant_w4g32
        q4.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
        q4.restype = C.c_int32
        q8 = lib.strata_b200_quant_w8pc
        q8.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
        q8.restype = C.c_int32
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev)
        gen.manual_seed(1234 + rank)
        self.tensors, self.arena, self.bufs = {}, {}, []
        stream = torch.cuda.current_stream().cuda_stream
        for i, v in enumerate(g.values):
            if v.producer is not None:
                continue
            if v.dtype.element == 10:  # int4 codes: quantise N(0, 0.02) f32 on the device
                n, kh = v.dims
                w = torch.randn((n, kh * 2), generator=gen, device=dev, dtype=torch.float32) * 0.02
                codes = torch.empty((n, kh), dtype=torch.uint8, device=dev)
                scales = torch.empty((n, kh * 2 // 32), dtype=torch.int16, device=dev)
                rc = q4(w.data_ptr(), n, kh * 2, codes.data_ptr(), scales.data_ptr(), stream)
                assert rc == 0, rc
                del w
                self.tensors[i], self.tensors[i + 1] = codes, scales
            elif v.dtype.element == 6:  # int8 codes: quantise N(0, 0.02) f32 per output channel
                n, k = v.dims
                w = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32) * 0.02
                codes = torch.empty((n, k), dtype=torch.int8, device=dev)
                scales = torch.empty((n,), dtype=torch.float32, device=dev)
                rc = q8(w.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(), stream)
                assert rc == 0, rc
                del w
                self.tensors[i], self.tensors[i + 1] = codes, scales
            elif i in self.tensors:
                continue
            elif v.dtype.element == 8:  # ids / positions
                self.tensors[i] = torch.zeros(v.dims, dtype=torch.int32, device=dev)
            elif v.name.endswith("cache"):
                c = torch.zeros(v.dims, dtype=torch.bfloat16, device=dev)
                if not prefill:
                    c[:, :, :kv_fill].normal_(generator=gen)
                self.tensors[i] = c
            elif "norm" in v.name:
                self.tensors[i] = (1 + 0.02 * torch.randn(v.dims, generator=gen, device=dev)).to(torch.bfloat16)
            else:
                self.tensors[i] = torch.randn(v.dims, generator=gen, device=dev).to(torch.bfloat16)
        torch.cuda.synchronize()
        if kv_page:  # every sequence's pages scattered over the pool in a seeded order
            n = self.tensors[hd.block_table].numel()
            perm = torch.randperm(n, generator=gen, device=dev).to(torch.int32)
            self.tensors[hd.block_table].copy_(perm.view(self.tensors[hd.block_table].shape))
        if prefill:  # each prompt from position 0
            self.tensors[hd.pos].copy_(torch.arange(seq, device=dev, dtype=torch.int32).repeat(batch))
        else:
            self.tensors[hd.pos].fill_(kv_fill)
        if self.embed:
            ids = torch.randint(0, shape.vocab, (batch * seq,), generator=gen, device=dev, dtype=torch.int32)
            self.tensors[hd.tokens].copy_(ids)
        for i, t in self.tensors.items():
            b = plugin.wrap(t.data_ptr(), t.numel() * t.element_size())
            self.bufs.append(b)
            self.arena[i] = Device(b)
        self.exe = plugin.compile(g)
        if self.exe is None:
            raise RuntimeError("the plugin declined the step")
        self.bound = self.exe.bind(self.arena)
        self.ids_buf = self.arena[hd.tokens].buffer
        self.pos_buf = self.arena[hd.pos].buffer
        self.out_buf = self.bound.outputs[hd.out]

    def close(self):
        self.bound.release()
        self.exe.free()
        for b in self.bufs:
            b.release()
        self.tensors.clear()


def dominant_kernel(plugin, torch, shape=LLAMA_7B, m=1, tp=1, reps=32):
    """Time the gate/up + SwiGLU int4 GEMV launch (the largest weight stream of
    the step) over `reps` distinct weight sets (more bytes than L2 holds), on
    the plugin's stream: x [m, hidden], one tensor-parallel shard's rows."""
    from strata_host import BF16, W4G32, Device, GraphBuilder, Op
    D, F = shape.hidden, ffn_shard(shape.ffn, tp, 0)[1]
    reps = max(2, min(reps, int(2.5e9 // (F * D))))
    b = GraphBuilder("gateup")
    x = b.input(BF16, (m, D), "x")
    outs = []
    for i in range(reps):
        wg, sg = b.input(W4G32, (F, D // 2), f"wg{i}"), b.input(BF16, (F, D // 32), f"sg{i}")
        wu, su = b.input(W4G32, (F, D // 2), f"wu{i}"), b.input(BF16, (F, D // 32), f"su{i}")
        g_ = b.node(Op.custom("fused::linear_w4g32"), [x, wg, sg], [(BF16, (m, F))], {}, f"g{i}")[0]
        u_ = b.node(Op.custom("fused::linear_w4g32"), [x, wu, su], [(BF16, (m, F))], {}, f"u{i}")[0]
        s_ = b.node(Op.custom("fused::swiglu"), [g_, u_], [(BF16, (m, F))], {}, f"s{i}")[0]
        outs.append(s_)
    for o in outs:
        b.output(o)
    g = b.build()
    dev = torch.device("cuda", torch.cuda.current_device())
    tensors, arena, bufs = [], {}, []
    for i, v in enumerate(g.values):
        if v.producer is None:
            t = torch.randint(0, 255, v.dims, dtype=torch.uint8, device=dev) if v.dtype == W4G32 else \
                (torch.rand(v.dims, device=dev) * 0.01).to(torch.bfloat16)
            tensors.append(t)
            bb = plugin.wrap(t.data_ptr(), t.numel() * t.element_size())
            bufs.append(bb)
            arena[i] = Device(bb)
    exe = plugin.compile(g)
    bound = exe.bind(arena)
    stream = torch.cuda.ExternalStream(plugin.stream())
    for _ in range(3):
        bound.run_async()
    plugin.synchronize()
    iters = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        bound.run_async()
    e1.record(stream)
    plugin.synchronize()
    per_launch_s = e0.elapsed_time(e1) / 1e3 / (iters * reps)
    bytes_per_launch = 2 * (F * D // 2 + F * (D // 32) * 2) + m * (D * 2 + F * 2)
    bound.release()
    exe.free()
    for bb in bufs:
        bb.release()
    return per_launch_s, bytes_per_launch


_CPU_INPUTS: dict = {}


def _cpu_inputs(shape, batch, kv_fill):
    """Host inputs for the CPU oracle's decode step, generated once: one
    layer's int4 weights (every layer runs on them: the oracle's time does
    not depend on the values, and 32 distinct layers would need 26 GB of f32
    to generate), norm gains, one KV cache pair prefilled over kv_fill
    positions, the embedding table and the int4 lm_head."""
    import numpy as np

    from oracle import oracle as ora
    key = (shape, batch, kv_fill)
    if key in _CPU_INPUTS:
        return _CPU_INPUTS[key]
    D, H, G, d, F, V = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn, shape.vocab
    mats = {"q": (H * d, D), "k": (G * d, D), "v": (G * d, D), "o": (D, H * d), "g": (F, D), "u": (F, D),
            "d": (D, F)}
    W = {k: ora.quant_w4g32(ora.normal(10 + i, (n, kk), std=0.02)) for i, (k, (n, kk)) in enumerate(mats.items())}
    kc = ora.round_bf16(ora.normal(20, (batch, G, kv_fill + 1, d)))
    vc = ora.round_bf16(ora.normal(21, (batch, G, kv_fill + 1, d)))
    norms = [ora.round_bf16(1.0 + ora.normal(30 + i, (D,), std=0.02)) for i in range(3)]
    table = ora.round_bf16(ora.normal(40, (V, D))) if V else None
    lm = ora.quant_w4g32(ora.normal(99, (V, D), std=0.02)) if V else None
    ids = ora.uniform_i32(2, batch, 0, V) if V else None
    h0 = ora.round_bf16(ora.normal(0, (batch, D)))
    _CPU_INPUTS[key] = (W, kc, vc, norms, table, lm, ids, h0)
    return _CPU_INPUTS[key]


def cpu_decode_layers(shape, batch, kv_fill, threads, layers, head=True):
    """One decode step on the CPU oracle: `layers` decoder layers (RMSNorm,
    q/k/v int4 linears, RoPE, KV append, attention over kv_fill + 1
    positions, o_proj + residual, RMSNorm, gate/up, SwiGLU, down_proj +
    residual) and, with `head`, the final norm, the int4 lm_head and argmax.
    Every value is rounded to bf16 where the graph produces it, as the
    graph-level oracle does.  Returns the seconds it took."""
    import numpy as np

    from oracle import oracle as ora
    W, kc, vc, norms, table, lm, ids, h0 = _cpu_inputs(shape, batch, kv_fill)
    H, G, d = shape.heads, shape.kv_heads, shape.head_dim
    r = ora.round_bf16
    pos = np.full(batch, kv_fill, np.int32)
    seq = np.arange(batch, dtype=np.int32)

    def lin(x, k):
        return r(ora.linear_w4g32(x, W[k][0], W[k][1], threads=threads))

    t0 = time.perf_counter()
    h = r(ora.embed(ids, table)[0]) if table is not None else h0
    for _ in range(layers):
        n = r(ora.rms_norm(h, norms[0], shape.eps))
        q = r(ora.rope(lin(n, "q"), pos, d, shape.theta))
        k = r(ora.rope(lin(n, "k"), pos, d, shape.theta))
        v = lin(n, "v")
        kc[:, :, kv_fill] = k.reshape(batch, G, d)
        vc[:, :, kv_fill] = v.reshape(batch, G, d)
        a = r(ora.attention(q, kc, vc, seq, pos, H, G, d, threads=threads))
        h = r(h + lin(a, "o"))
        n = r(ora.rms_norm(h, norms[1], shape.eps))
        gu = r(ora.swiglu(lin(n, "g"), lin(n, "u")))
        h = r(h + lin(gu, "d"))
    if head and lm is not None:
        n = r(ora.rms_norm(h, norms[2], shape.eps))
        ora.argmax(r(ora.linear_w4g32(n, lm[0], lm[1], threads=threads)))
    return time.perf_counter() - t0


def cpu_step_sample(shape, batch, kv_fill, threads, whole_step=True):
    """The CPU baseline beside the B200 arm: one whole decode step on all host
    threads (or, for a stack too large to run whole in a few minutes, one
    layer scaled to the stack), and one layer on one thread scaled to the
    stack (the reference's own CPU backend is single-threaded)."""
    head = "the int4 lm_head and argmax" if shape.vocab else "no lm_head"
    if whole_step:
        step_s = cpu_decode_layers(shape, batch, kv_fill, threads, shape.layers)
        what = f"one whole decode step at batch {batch} ({shape.layers} layers over {kv_fill + 1} positions, {head})"
    else:
        step_s = cpu_decode_layers(shape, batch, kv_fill, threads, 1, head=False) * shape.layers
        what = (f"one decode layer at batch {batch} over {kv_fill + 1} positions, scaled x{shape.layers} "
                f"(an extrapolation; {head})")
    one = cpu_decode_layers(shape, batch, kv_fill, 1, 1, head=False)
    return {"value": batch / step_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{what} on the threaded C oracle; every layer reuses one layer's weights",
            "single_thread": {"value": batch / (one * shape.layers), "unit": "tokens/s", "cores": 1,
                              "sample": f"one layer on one thread, scaled x{shape.layers} (lm_head excluded)"}}


def decode_config(args, shape, kv_fill, world, sb):
    """The `config` object both arms print for the decode workload."""
    head = "int4 lm_head + argmax" if shape.vocab else "no embedding / lm_head"
    return {"workload": f"{args.model.upper()}-shape int4 g32 decode stack ({args.layers} layers, "
                        f"{head}), batch {args.batch}, KV cache {kv_fill} prefilled",
            "model": args.model, "batch": args.batch, "kv_len": kv_fill, "layers": args.layers,
            "parallelism": f"tp{world}",
            "kv_cache": f"paged, {args.kv_page}-position pages" if args.kv_page else "contiguous",
            "l2": f"inputs larger than L2: {sb / 1e9:.2f} GB streamed per step"}


def run_reference(args):
    """The reference arm: the CPU oracle (the port of the reference's CPU
    backend plus the decoder ops it lacks) running whole decode steps of the
    same workload on all host threads.  Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as ora
    threads = ora.max_threads()
    shape, _, kv_fill, metric = MODELS[args.model]
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    steps = []
    for i in range(args.warmup + args.steps):
        t = cpu_decode_layers(shape, args.batch, kv_fill, threads, args.layers)
        if i >= args.warmup:
            steps.append(t)
    step_s = sum(steps) / len(steps)
    v = args.batch / step_s
    sb = step_bytes(shape, args.batch, kv_fill) * args.layers // shape.layers
    sample = (f"whole decode steps at batch {args.batch} ({args.layers} layers over {kv_fill + 1} positions"
              f"{', the int4 lm_head and argmax' if shape.vocab else ''}) on the threaded C oracle; every layer "
              f"reuses one layer's weights")
    line = {"impl": "reference", "metric": metric, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights (g32, bf16 scales), bf16-rounded values, f32 compute",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV)",
            "config": decode_config(args, shape, kv_fill, world, sb),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


PREFILL_METRIC = "prefill tokens/s, 7B-shape int8 per-channel stack"


def prefill_flops(shape, batch, seq, layers):
    """FLOPs of one prefill step: the linears (2 M K N each), causal attention
    (QK^T and PV over positions 0..t for each token t), the last-token lm_head."""
    D, H, G, d, F = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn
    M = batch * seq
    lin = 2 * M * (D * H * d + 2 * D * G * d + H * d * D + 2 * D * F + F * D) * layers
    attn = 2 * 2 * batch * H * d * (seq * (seq + 1) // 2) * layers
    return lin + attn + 2 * batch * D * shape.vocab


def run_prefill(args):
    """Config 4: batch x seq prompt tokens through every layer (int8 per-channel
    linears on the tcgen05 GEMM, causal prefill attention), logits for each
    sequence's last position."""
    import torch
    from strata_host import Plugin
    torch.cuda.set_device(0)
    plugin = Plugin(os.path.join(PKG, "libstrata_b200.so"))
    model = Model(plugin, torch, args.batch, 0, 1, args.layers, fmt="w8pc", seq=args.seq, head="logits")
    stream = torch.cuda.ExternalStream(plugin.stream())

    def sync():
        torch.cuda.synchronize()
        plugin.synchronize()

    for _ in range(args.warmup):
        model.bound.run_async()
    sync()
    if args.profile_step:
        torch.cuda.profiler.start()
        for _ in range(args.steps):
            model.bound.run_async()
        sync()
        torch.cuda.profiler.stop()
        model.close()
        plugin.close()
        return 0
    launches0 = plugin.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        sync()
        e0.record(stream)
        for _ in range(args.steps):
            model.bound.run_async()
        e1.record(stream)
        sync()
    launches = plugin.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    tokens = args.batch * args.seq
    # End to end: ids and positions from pinned host memory in, last-token logits out.
    n_in = tokens * 4
    ids_h = torch.randint(0, LLAMA_7B.vocab, (tokens,), dtype=torch.int32).pin_memory()
    pos_h = torch.arange(args.seq, dtype=torch.int32).repeat(args.batch).pin_memory()
    out_b = model.bound.outputs[model.hd.out]
    n_out = args.batch * LLAMA_7B.vocab * 2
    out_h = torch.empty(n_out, dtype=torch.uint8).pin_memory()

    def e2e_step():
        model.ids_buf.write_ptr(ids_h.data_ptr(), n_in)
        model.pos_buf.write_ptr(pos_h.data_ptr(), n_in)
        model.bound.run()
        out_b.read_into(out_h.data_ptr(), n_out)

    e2e_step()
    sync()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    sync()
    e2e_s = (time.perf_counter() - t0) / args.steps
    flops = prefill_flops(LLAMA_7B, args.batch, args.seq, args.layers)
    try:
        with open(PEAKS_PATH) as f:
            peak, peak_kind = float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        peak, peak_kind = 1400.0, "fallback (sustained)"
    tf = flops / (ms / 1e3) / 1e12
    line = {
        "metric": PREFILL_METRIC, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 weights (per-channel f32 scale), bf16 activations, f32 accumulate",
        "data": "synthetic: device-generated N(0,0.02) weights quantised by the plugin, uniform token ids",
        "config": {"workload": f"7B-shape int8 prefill ({args.layers} layers), batch {args.batch} x "
                               f"{args.seq} tokens, logits for the last position only",
                   "batch": args.batch, "seq_len": args.seq, "layers": args.layers, "parallelism": "tp1",
                   "l2": "inputs larger than L2"},
        "e2e": {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 2 * n_in,
                "d2h_bytes_per_step": n_out},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                     "peak_kind": peak_kind, "flops_per_step": flops},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line))
    model.close()
    plugin.close()
    return 0


SWEEP_METRIC = "quantized Linear sweep, K = N = 4096 (us per launch, % of roofline)"


def run_sweep(args):
    """Config 2: one quantized Linear node per case, int4 g32 and int8 per-channel weights
    (plus MXFP8 / MXFP4 weights with E8M0 block scales), K = N = 4096, M in {1, 16, 128, 2048},
    through the C-ABI entry points (strata_b200_linear_w4g32 / _w8pc / _mxfp8 / _mxfp4: the
    tensor-core GEMV up to 64 rows, the tcgen05 GEMM above).  Weight copies rotate so every
    launch streams its weights from HBM."""
    import torch
    torch.cuda.set_device(0)
    lib = C.CDLL(os.path.join(PKG, "libstrata_b200.so"))
    P, I64 = C.c_void_p, C.c_int64
    for f in (lib.strata_b200_linear_w4g32, lib.strata_b200_linear_w8pc, lib.strata_b200_linear_mxfp8,
              lib.strata_b200_linear_mxfp4):
        f.argtypes = [P, I64, I64, P, P, I64, P, P, P]
        f.restype = C.c_int32
    bw, bw_kind = load_peaks()
    try:
        with open(PEAKS_PATH) as fh:
            tf_peak, tf_kind = float(json.load(fh)["bf16_tflops"]), "measured (burst)"
    except Exception:
        tf_peak, tf_kind = 1590.0, "fallback (burst)"
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    K = N = 4096
    stream = torch.cuda.current_stream()
    cases = []
    for fmt in ("w4g32", "w8pc", "mxfp8", "mxfp4"):
        wbytes = {"w4g32": N * K // 2 + N * (K // 32) * 2, "w8pc": N * K + N * 4,
                  "mxfp8": N * K + N * (K // 32), "mxfp4": N * K // 2 + N * (K // 32)}[fmt]
        copies = max(2, (2 * l2) // wbytes + 1)
        if fmt == "w4g32":
            ws = [torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda") for _ in range(copies)]
            ss = [(torch.rand((N, K // 32), device="cuda") * 0.01).to(torch.bfloat16) for _ in range(copies)]
            fn = lib.strata_b200_linear_w4g32
        elif fmt in ("mxfp8", "mxfp4"):  # random finite codes, E8M0 scales around 2^-7
            cb = K if fmt == "mxfp8" else K // 2
            ws = [torch.randint(0, 256, (N, cb), dtype=torch.uint8, device="cuda") for _ in range(copies)]
            if fmt == "mxfp8":  # no NaN codes (0x7f / 0xff)
                for w_ in ws:
                    w_[(w_ & 0x7F) == 0x7F] = 0
            ss = [torch.randint(110, 130, (N, K // 32), dtype=torch.uint8, device="cuda") for _ in range(copies)]
            fn = lib.strata_b200_linear_mxfp8 if fmt == "mxfp8" else lib.strata_b200_linear_mxfp4
        else:
            ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda") for _ in range(copies)]
            ss = [torch.rand((N,), device="cuda") * 0.01 for _ in range(copies)]
            fn = lib.strata_b200_linear_w8pc
        for m in (1, 16, 128, 2048):
            x = torch.randn((m, K), device="cuda").to(torch.bfloat16)
            y = torch.empty((m, N), dtype=torch.bfloat16, device="cuda")

            def launch(i):
                rc = fn(x.data_ptr(), m, K, ws[i % copies].data_ptr(), ss[i % copies].data_ptr(), N, None,
                        y.data_ptr(), stream.cuda_stream)
                assert rc == 0, rc

            for i in range(max(args.warmup, 3) * copies):
                launch(i)
            torch.cuda.synchronize()
            reps = max(args.steps, 1) * copies
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(reps):
                launch(i)
            e1.record(stream)
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / 1e3 / reps
            nbytes = wbytes + m * K * 2 + m * N * 2
            flops = 2 * m * N * K
            t_roof = max(nbytes / (bw * 1e9), flops / (tf_peak * 1e12))
            bound = "hbm" if nbytes / (bw * 1e9) >= flops / (tf_peak * 1e12) else "tensor"
            cases.append({"fmt": fmt, "m": m, "us": t * 1e6, "bytes": nbytes, "flops": flops,
                          "gbs": nbytes / t / 1e9, "tflops": flops / t / 1e12, "bound": bound,
                          "frac": t_roof / t})
        del ws, ss
        torch.cuda.empty_cache()
    line = {"metric": SWEEP_METRIC, "value": cases[0]["frac"], "unit": "fraction of roofline (int4, M=1)",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 g32 / int8 per-channel weights, bf16 activations, f32 accumulate",
            "data": "synthetic: random codes and scales on the device, N(0,1) bf16 x",
            "config": {"workload": "one quantized Linear node, K = N = 4096, M in {1, 16, 128, 2048}",
                       "l2": f"{copies}+ weight copies rotated (more than twice the {l2 >> 20} MB L2)"},
            "roofline": {"hbm_gbs": bw, "hbm_kind": bw_kind, "bf16_tflops": tf_peak, "tensor_kind": tf_kind},
            "cases": cases}
    print(json.dumps(line))
    return 0


def run_breakdown(args, plugin, model, shape, kv_fill, world, rank, barrier):
    """Per step-class device time of the decode step: every run is eager and
    each step is bracketed by CUDA events on the plugin's stream (so the
    classes' times add up to a little more than the graph-replayed step,
    which overlaps neighbouring kernels).  The maximum over ranks per class."""
    import torch
    import torch.distributed as dist
    lib = C.CDLL(plugin.path)
    fn = lib.strata_b200_step_times
    fn.argtypes = [C.c_char_p, C.c_uint64, C.c_int32]
    fn.restype = C.c_uint64
    for _ in range(args.warmup):
        model.bound.run()
    barrier()
    fn(None, 0, 1)  # reset
    for _ in range(args.steps):
        model.bound.run()
    barrier()
    buf = C.create_string_buffer(int(fn(None, 0, 0)) + 1)
    fn(buf, len(buf), 1)
    mine = {k: (v[0] / args.steps, v[1] * 1e3 / args.steps) for k, v in json.loads(buf.value.decode()).items()}
    every = [mine]
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, mine)
    if rank == 0:
        classes = sorted({k for d in every for k in d})
        out = {k: {"steps_per_step": max(d.get(k, (0, 0))[0] for d in every),
                   "us_per_step": round(max(d.get(k, (0, 0))[1] for d in every), 2)} for k in classes}
        total = sum(v["us_per_step"] for v in out.values())
        print(json.dumps({"metric": "decode step breakdown (eager, CUDA events between steps)",
                          "unit": "us per step, max over ranks", "n_gpus": world, "steps": args.steps,
                          "config": decode_config(args, shape, kv_fill, world,
                                                  step_bytes(shape, args.batch, kv_fill) * args.layers // shape.layers),
                          "classes": dict(sorted(out.items(), key=lambda kv: -kv[1]["us_per_step"])),
                          "sum_us_per_step": round(total, 1)}))
    model.close()
    plugin.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--model", default="7b", choices=sorted(MODELS),
                    help="7b: 7B-shape stack (default batch 8, KV 2048); 70b: 70B-shape stack (batch 32, KV 4096)")
    ap.add_argument("--batch", type=int, default=None, help="sequences per step (default: per --model)")
    ap.add_argument("--layers", type=int, default=None, help="layers (default: all of --model's)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill", action="store_true",
                    help="time the int8 prefill configuration instead of decode")
    ap.add_argument("--seq", type=int, default=2048, help="tokens per prompt with --prefill")
    ap.add_argument("--sweep", action="store_true",
                    help="time the quantized Linear sweep (K = N = 4096, M in {1, 16, 128, 2048}, "
                         "int4, int8, MXFP8, MXFP4)")
    ap.add_argument("--breakdown", action="store_true",
                    help="instead of the timed run: device time per step class (GEMVs, attention, "
                         "all-reduce + add + norm, ...) of the decode step, run eagerly with CUDA events "
                         "between steps; under torchrun rank 0 prints the maximum over ranks")
    ap.add_argument("--kv-page", type=int, default=0,
                    help="decode with a paged KV cache of this page size (block table, shuffled pages)")
    ap.add_argument("--profile-step", action="store_true",
                    help="after the warm-up, run --steps steps between cudaProfilerStart/Stop and exit "
                         "(for ncu --profile-from-start off)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    shape, batch0, kv_fill, metric = MODELS[args.model]
    if args.batch is None:
        args.batch = batch0
    if args.layers is None:
        args.layers = shape.layers
    if args.prefill and args.model != "7b":
        ap.error("--prefill runs the 7B-shape int8 configuration only")
    if args.impl == "reference":
        return run_reference(args)
    if args.prefill:
        return run_prefill(args)
    if args.sweep:
        return run_sweep(args)

    import torch
    import torch.distributed as dist
    from strata_host import Plugin

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    os.environ["STRATA_B200_DEVICE"] = str(local)
    if args.breakdown:
        os.environ["STRATA_B200_STEP_TIMES"] = "1"  # read once, when the library loads
    plugin = Plugin(os.path.join(PKG, "libstrata_b200.so"))
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(plugin.tp_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        plugin.tp_init(rank, world, bytes(uid.cpu().numpy().tobytes()))

    model = Model(plugin, torch, args.batch, rank, world, args.layers, shape=shape, kv_fill=kv_fill,
                  kv_page=args.kv_page)
    stream = torch.cuda.ExternalStream(plugin.stream())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        plugin.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.breakdown:
        return run_breakdown(args, plugin, model, shape, kv_fill, world, rank, barrier)

    # ---- device-timed steps (inputs resident, CUDA-graph replay) -------------
    for _ in range(args.warmup):
        model.bound.run_async()
    barrier()
    if args.profile_step:
        # --steps steps between cudaProfilerStart and cudaProfilerStop, for a
        # profiler started with --profile-from-start off; nothing else runs.
        torch.cuda.profiler.start()
        for _ in range(args.steps):
            model.bound.run_async()
        barrier()
        torch.cuda.profiler.stop()
        model.close()
        plugin.close()
        if world > 1:
            dist.destroy_process_group()
        return 0
    launches0 = plugin.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            model.bound.run_async()
        e1.record(stream)
        barrier()
    launches = plugin.launch_count() - launches0
    dev_s = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    ms_step = dev_s / args.steps * 1e3
    tokens = args.batch * args.steps
    value = tokens / dev_s

    # ---- end to end through the ABI with host buffers ------------------------
    # Token ids (or, without an embedding, the bf16 hidden states) and the
    # positions in; the next ids (or the last hidden states) out.
    pos_h = torch.full((args.batch,), kv_fill, dtype=torch.int32).pin_memory()
    if model.embed:
        ids_h = torch.zeros(args.batch, dtype=torch.int32).pin_memory()
        out_h = torch.zeros(args.batch, dtype=torch.int32).pin_memory()
    else:
        ids_h = torch.randn((args.batch, shape.hidden)).to(torch.bfloat16).pin_memory()
        out_h = torch.zeros((args.batch, shape.hidden), dtype=torch.bfloat16).pin_memory()
    n_in = ids_h.numel() * ids_h.element_size()
    n_out = out_h.numel() * out_h.element_size()
    nb = args.batch * 4

    def e2e_step():
        model.ids_buf.write_ptr(ids_h.data_ptr(), n_in)
        model.pos_buf.write_ptr(pos_h.data_ptr(), nb)
        model.bound.run()
        model.out_buf.read_into(out_h.data_ptr(), n_out)
        if model.embed:
            ids_h.copy_(out_h)  # feed the predicted ids back as the next tokens

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    t_wall = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    f1.record(stream)
    barrier()
    wall = time.perf_counter() - t_wall
    e2e_s = max_over_ranks(max(f0.elapsed_time(f1) / 1e3, wall))
    e2e = tokens / e2e_s

    # ---- roofline of the dominant kernel and of the whole step ----------------
    # The dominant kernel is timed at the step's own M (the batch) and, as a
    # side figure, at M = 1.
    peak, peak_kind = load_peaks()
    k_m = args.batch
    k_s, k_bytes = dominant_kernel(plugin, torch, shape=shape, m=k_m, tp=world)
    k_gbs = k_bytes / k_s / 1e9
    k1_s, k1_bytes = dominant_kernel(plugin, torch, shape=shape, m=1, tp=world) if k_m != 1 else (k_s, k_bytes)
    sb = step_bytes(shape, args.batch, kv_fill) * args.layers // shape.layers
    step_gbs = sb / (ms_step / 1e3) / 1e9 / world
    clock = clocks.summary()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as ora
        cpu = cpu_step_sample(shape, args.batch, kv_fill, ora.max_threads(), whole_step=args.model == "7b")

    if rank == 0:
        F = ffn_shard(shape.ffn, world, 0)[1]
        line = {
            "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights (g32, bf16 scales), bf16 activations, f32 accumulate",
            "data": "synthetic: device-generated N(0,0.02) weights quantised by the plugin, N(0,1) bf16 KV",
            "config": decode_config(args, shape, kv_fill, world, sb),
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": n_in + nb, "d2h_bytes_per_step": n_out},
            "roofline": {"bound": "hbm",
                         "kernel": f"w4g32 gate/up GEMV + SwiGLU epilogue, M={k_m}, N=2x{F}, K={shape.hidden}",
                         "achieved": k_gbs, "peak": peak, "unit": "GB/s", "frac": k_gbs / peak,
                         "peak_kind": peak_kind,
                         "traffic": measured_traffic(k_m, 2 * F, shape.hidden),
                         "bytes_per_launch": k_bytes, "us_per_launch": k_s * 1e6,
                         "m1": {"achieved": k1_bytes / k1_s / 1e9, "frac": k1_bytes / k1_s / 1e9 / peak,
                                "bytes_per_launch": k1_bytes, "us_per_launch": k1_s * 1e6,
                                "traffic": measured_traffic(1, 2 * F, shape.hidden)}},
            "step_roofline": {"bytes_per_step": sb, "achieved_gbs_per_gpu": step_gbs, "frac": step_gbs / peak,
                              "frac_of_8tbs": step_gbs / 8000.0},
            "gpu_launches": launches,
            "clocks": clock,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line))
    model.close()
    plugin.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
