"""Graph-level parity on the B200 through the plugin ABI (strata_plugin_v1):
compile a subgraph, run it with device buffers, compare with the oracle."""
import json
import os

import numpy as np
import pytest

from oracle import graph_eval, oracle as ora
from strata_host import BF16, F32, I32, W4G32, Device, GraphBuilder, Op, StrataError, w8pc
from strata_host.blocks import BLOCK_512, LLAMA_7B, LLAMA_70B, DecoderShape, decoder_graph
from tests.helpers import TOL_BF16, TOL_F32, assert_close, seeded_graph_inputs, to_device_bytes

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")


def run_graph(plugin, graph, host_vals, every_value=False):
    """Upload every input as a device-resident buffer, run, return outputs."""
    arena = {}
    bufs = []
    for i, v in enumerate(graph.values):
        if v.producer is None and i in host_vals:
            b = plugin.upload(v.dtype, v.dims, to_device_bytes(v, host_vals[i]))
            bufs.append(b)
            arena[i] = Device(b)
    exe = plugin.compile(graph)
    assert exe is not None, "the plugin declined a hot-path graph"
    try:
        exe.run(arena, every_value=every_value)
        out = {o: arena[o] for o in graph.outputs}
        caches = {i: bytes(arena[i].buffer.read()) for i, v in enumerate(graph.values)
                  if v.name.endswith("cache") and i in arena}
    finally:
        for b in bufs:
            b.release()
        exe.free()
    return out, caches


def as_f32(v, arr):
    if v.dtype == BF16:
        return ora.from_bf16(np.asarray(arr).view(np.uint16))
    return np.asarray(arr)


@pytest.mark.parametrize("case", json.load(open(GOLDEN)), ids=lambda c: c["id"])
def test_reference_known_answers_through_the_plugin(cuda, plugin, case):
    """kernels.rs / end_to_end.rs golden values, run as one-node f32 graphs."""
    b = GraphBuilder(case["id"])
    op = case["op"]
    host = {}
    arr = lambda k: np.array(case[k], np.float32)
    if op in ("add", "matmul"):
        a, c = arr("a"), arr("b")
        ia, ic = b.input(F32, a.shape, "a"), b.input(F32, c.shape, "b")
        host = {ia: a, ic: c}
        shape = tuple(case.get("out_shape") or (a.shape[0], c.shape[1]))
        out = b.node(Op(op), [ia, ic], [(F32, shape)], {}, "op0")[0]
    elif op in ("softmax", "gelu", "transpose", "expand"):
        x = arr("x")
        ix = b.input(F32, x.shape, "x")
        host = {ix: x}
        if op == "softmax":
            out = b.node(Op("softmax", axis=-1), [ix], [(F32, x.shape)], {}, "op0")[0]
        elif op == "gelu":
            out = b.node(Op("gelu"), [ix], [(F32, x.shape)], {}, "op0")[0]
        elif op == "transpose":
            out = b.node(Op("transpose", permutation=(1, 0)), [ix], [(F32, x.shape[::-1])], {}, "op0")[0]
        else:
            shape = tuple(case["out_shape"])
            out = b.node(Op("expand", shape=shape), [ix], [(F32, shape)], {}, "op0")[0]
    elif op == "layer_norm":
        x, g, be = arr("x"), arr("gamma"), arr("beta")
        ix, ig, ib = b.input(F32, x.shape, "x"), b.input(F32, g.shape, "gamma"), b.input(F32, be.shape, "beta")
        host = {ix: x, ig: g, ib: be}
        out = b.node(Op("layer_norm", gamma=ig, beta=ib, eps=case["eps"]), [ix], [(F32, x.shape)], {}, "ln0")[0]
    elif op == "linear":
        x, w = arr("x"), arr("w")
        ix, iw = b.input(F32, x.shape, "x"), b.input(F32, w.shape, "w")
        host = {ix: x, iw: w}
        ibias = None
        if case["bias"] is not None:
            ibias = b.input(F32, (w.shape[0],), "b")
            host[ibias] = arr("bias")
        out = b.node(Op("linear", weight=iw, bias=ibias), [ix], [(F32, (x.shape[0], w.shape[0]))], {}, "fc0")[0]
    elif op == "gelu_mul":
        x = arr("x")
        ix = b.input(F32, x.shape, "x")
        host = {ix: x}
        g = b.node(Op("gelu"), [ix], [(F32, x.shape)], {}, "gelu0")[0]
        out = b.node(Op("mul"), [g, ix], [(F32, x.shape)], {}, "mul0")[0]
    else:
        raise AssertionError(op)
    b.output(out)
    g = b.build()
    res, _ = run_graph(plugin, g, host, every_value=True)
    got = np.asarray(res[out]).ravel()
    if op == "gelu_mul":
        for v, w, t in zip(got[:2], case["want_first"], case["tol"]):
            assert abs(v - w) < t
    else:
        assert np.all(np.abs(got - np.array(case["want"], np.float32)) <= max(case["tol"], 1e-6)), got


def test_f32_llama_block_matches_oracle(cuda, plugin):
    """The single f32 decoder block: hidden 512, 8 x 64 MHA, FFN 1408, seq 128."""
    S = 128
    g, hd = decoder_graph(BLOCK_512, batch=1, seq=S, max_len=S, fmt="f32", embed=False, head="none")
    host = seeded_graph_inputs(g)
    host[hd.pos] = np.arange(S, dtype=np.int32)
    res, _ = run_graph(plugin, g, host)
    want = graph_eval.evaluate(g, dict(host))[hd.out]
    assert_close(res[hd.out], want, TOL_F32, "f32 block")


@pytest.mark.parametrize("fmt", ["w4g32", "w8pc"])
@pytest.mark.parametrize("m", [1, 16, 128])
def test_quantized_linear_node(cuda, plugin, fmt, m):
    k = n = 4096
    b = GraphBuilder("qlin")
    ix = b.input(BF16, (m, k), "x")
    if fmt == "w4g32":
        iw, is_ = b.input(W4G32, (n, k // 2), "w"), b.input(BF16, (n, k // 32), "s")
    else:
        iw, is_ = b.input(w8pc(k), (n, k), "w"), b.input(F32, (n,), "s")
    out = b.node(Op.custom(f"fused::linear_{fmt}"), [ix, iw, is_], [(BF16, (m, n))], {}, "lin")[0]
    b.output(out)
    g = b.build()
    host = seeded_graph_inputs(g)
    host[ix] = ora.round_bf16(ora.normal(0, (m, k)))
    res, _ = run_graph(plugin, g, host)
    want = graph_eval.evaluate(g, dict(host))[out]
    assert_close(as_f32(g.values[out], res[out]), want, TOL_BF16, f"{fmt} m={m}")


def _decode_case(plugin, shape, batch, layers, max_len, fill, tp_world=1, head="logits"):
    g, hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", layers=layers,
                          embed=shape.vocab > 0, head=head if shape.vocab else "none",
                          tp_world=tp_world)
    host = seeded_graph_inputs(g, cache_fill=fill)
    if shape.vocab:
        host[hd.tokens] = ora.uniform_i32(2, batch, 0, shape.vocab)
    else:
        host[hd.tokens] = ora.round_bf16(ora.normal(0, (batch, shape.hidden)))
    host[hd.pos] = np.array([fill - i for i in range(batch)], np.int32)
    res, caches = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in host.items()})
    return g, hd, res, caches, ref


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_llama7b_shape_decode_two_layers(cuda, plugin, batch):
    """7B-shape decode (int4 g32, KV 2048 prefilled) at reduced depth: 2 layers,
    at each batch of the decode configuration.  Batch 64 runs the GEMV's widest
    x-row blocks (33-64 rows) in the q/k/v + RoPE and gate/up + SwiGLU
    epilogues."""
    g, hd, res, caches, ref = _decode_case(plugin, LLAMA_7B, batch, 2, 2112, 2048)
    assert_close(as_f32(g.values[hd.out], res[hd.out]), ref[hd.out], TOL_BF16, "7B logits")
    for i, raw in caches.items():  # the appended k/v rows match the oracle's
        got = ora.from_bf16(np.frombuffer(raw, np.uint16).reshape(g.values[i].dims))
        assert_close(got, ref[i], TOL_BF16, g.values[i].name)


def test_llama7b_shape_argmax_is_exact_on_device_logits(cuda, plugin):
    g, hd = decoder_graph(LLAMA_7B, batch=4, seq=1, max_len=2112, fmt="w4g32", layers=1, head="argmax")
    logits_id = g.nodes[-1].inputs[0]
    g.outputs.append(logits_id)
    host = seeded_graph_inputs(g, cache_fill=2048)
    host[hd.tokens] = ora.uniform_i32(2, 4, 0, LLAMA_7B.vocab)
    host[hd.pos] = np.full(4, 2048, np.int32)
    res, _ = run_graph(plugin, g, host)
    logits = as_f32(g.values[logits_id], res[logits_id])
    assert np.array_equal(np.asarray(res[hd.out]), ora.argmax(logits))
    ref = graph_eval.evaluate(g, host)
    assert_close(logits, ref[logits_id], TOL_BF16, "lm_head logits")


@pytest.mark.parametrize("fmt,kv_heads", [("w8pc", 8), ("w4g32", 8), ("w8pc", 2)])
def test_prefill_runs_tensor_core_gemms_and_matches_oracle(cuda, plugin, fmt, kv_heads):
    """A prefill step (2 sequences x 96 tokens from position 0 = 192 rows): the
    linears run as tcgen05 GEMMs, rope / KV append as their own steps, causal
    attention on the prefill kernel (a partial second 64-row query tile; MHA and
    4:1 GQA).  A narrower decoder than 7B (hidden 1024, 8 heads x 128, FFN 2816)
    keeps the oracle's run short; the layer structure is the same."""
    shape = DecoderShape(1024, 8, kv_heads, 128, 2816, 512, 2)
    batch, seq = 2, 96
    g, hd = decoder_graph(shape, batch=batch, seq=seq, max_len=128, fmt=fmt, head="logits")
    host = seeded_graph_inputs(g, cache_fill=0)
    host[hd.tokens] = ora.uniform_i32(2, batch * seq, 0, shape.vocab)
    host[hd.pos] = np.tile(np.arange(seq, dtype=np.int32), batch)
    res, caches = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in host.items()})
    assert_close(as_f32(g.values[hd.out], res[hd.out]), ref[hd.out], TOL_BF16, f"prefill logits ({fmt})")
    for i, raw in caches.items():
        got = ora.from_bf16(np.frombuffer(raw, np.uint16).reshape(g.values[i].dims))
        assert_close(got, ref[i], TOL_BF16, g.values[i].name)


def test_llama7b_shape_int8_prefill_layer(cuda, plugin):
    """One 7B-shape int8 prefill layer at full width (hidden 4096, 32 x 128
    heads, FFN 11008, vocab 32000): 2 sequences x 128 tokens from position 0,
    so every linear is a tcgen05 GEMM (K = 11008 on down_proj, the SwiGLU
    epilogue at 11008 features) and the head runs on each sequence's last
    row."""
    batch, seq = 2, 128
    g, hd = decoder_graph(LLAMA_7B, batch=batch, seq=seq, max_len=seq, fmt="w8pc", layers=1, head="logits",
                          last_token=True)
    host = seeded_graph_inputs(g, cache_fill=0)
    host[hd.tokens] = ora.uniform_i32(2, batch * seq, 0, LLAMA_7B.vocab)
    host[hd.pos] = np.tile(np.arange(seq, dtype=np.int32), batch)
    res, caches = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in host.items()})
    assert g.values[hd.out].dims == (batch, LLAMA_7B.vocab)
    assert_close(as_f32(g.values[hd.out], res[hd.out]), ref[hd.out], TOL_BF16, "7B int8 prefill logits")
    for i, raw in caches.items():
        got = ora.from_bf16(np.frombuffer(raw, np.uint16).reshape(g.values[i].dims))
        assert_close(got, ref[i], TOL_BF16, g.values[i].name)


def test_loaded_executable_runs_on_the_device(cuda, plugin):
    """serialize -> deserialize_load -> run (raw.rs:760-788): an executable
    loaded from its blob runs a 7B-shape decode layer on the device and
    matches both the oracle and the executable it was saved from, bit for
    bit."""
    g, hd = decoder_graph(LLAMA_7B, batch=4, seq=1, max_len=2112, fmt="w4g32", layers=1, head="logits")
    host = seeded_graph_inputs(g, cache_fill=2048)
    host[hd.tokens] = ora.uniform_i32(2, 4, 0, LLAMA_7B.vocab)
    host[hd.pos] = np.array([2048, 2047, 1000, 3], np.int32)
    exe = plugin.compile(g)
    assert exe is not None
    blob = plugin.serialize(exe)
    exe.free()
    assert plugin.abi_compatible(blob)
    outs = []
    for loaded in (False, True):
        arena, bufs = {}, []
        for i, v in enumerate(g.values):
            if v.producer is None:
                b = plugin.upload(v.dtype, v.dims, to_device_bytes(v, host[i]))
                bufs.append(b)
                arena[i] = Device(b)
        e = plugin.deserialize(blob, g) if loaded else plugin.compile(g)
        try:
            e.run(arena, every_value=False)
            outs.append(arena[hd.out])
        finally:
            for b in bufs:
                b.release()
            e.free()
    assert np.array_equal(np.asarray(outs[0]), np.asarray(outs[1]))
    ref = graph_eval.evaluate(g, host)
    assert_close(as_f32(g.values[hd.out], outs[1]), ref[hd.out], TOL_BF16, "loaded executable logits")


@pytest.mark.parametrize("batch,seq,heads,kv_heads,d,offset", [
    (2, 300, 8, 2, 128, 0),     # 3 query tiles x 3 position tiles, 4:1 GQA
    (1, 520, 4, 4, 128, 0),     # 5 x 5 tiles, MHA, a 8-row last query tile
    (2, 200, 8, 8, 64, 0),      # head_dim 64
    (2, 150, 8, 4, 128, 333),   # continuing prompts: positions 333.. after a prefilled cache
])
def test_prefill_attention_kernel_across_tiles(cuda, plugin, batch, seq, heads, kv_heads, d, offset):
    """One fused::attention node over several tokens per sequence: the
    tcgen05 prefill kernel (128-row query tiles, 128-position K/V tiles,
    online softmax across tiles, causal mask from the positions) against the
    oracle, including a cache prefilled before the prompt's own positions."""
    b = GraphBuilder("prefill_attention")
    R, L = batch * seq, offset + seq + 37
    q = b.input(BF16, (R, heads * d), "q")
    k = b.input(BF16, (R, kv_heads * d), "k")
    v = b.input(BF16, (R, kv_heads * d), "v")
    kc = b.input(BF16, (batch, kv_heads, L, d), "k_cache")
    vc = b.input(BF16, (batch, kv_heads, L, d), "v_cache")
    pos = b.input(I32, (R,), "pos")
    out = b.node(Op.custom("fused::attention"), [q, k, v, kc, vc, pos], [(BF16, (R, heads * d))],
                 {"num_heads": heads, "num_kv_heads": kv_heads, "head_dim": d}, "attention")[0]
    b.output(out)
    g = b.build()
    cache = lambda seed: np.concatenate(
        [ora.round_bf16(ora.normal(seed, (batch, kv_heads, offset, d))),
         np.zeros((batch, kv_heads, L - offset, d), np.float32)], axis=2)
    host = {q: ora.round_bf16(ora.normal(51, (R, heads * d))), k: ora.round_bf16(ora.normal(52, (R, kv_heads * d))),
            v: ora.round_bf16(ora.normal(53, (R, kv_heads * d))), kc: cache(54), vc: cache(55),
            pos: np.tile(np.arange(offset, offset + seq, dtype=np.int32), batch)}
    res, caches = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {kk: (vv.copy() if isinstance(vv, np.ndarray) else vv) for kk, vv in host.items()})
    assert_close(as_f32(g.values[out], res[out]), ref[out], TOL_BF16, "prefill attention")


def test_prefill_last_token_head_runs_on_each_sequence_last_row(cuda, plugin):
    """fused::last_token: the prefill head (final norm, lm_head, argmax) runs on
    each sequence's last row only, giving the next token of every prompt."""
    shape = DecoderShape(1024, 8, 8, 128, 2816, 512, 1)
    batch, seq = 3, 80
    g, hd = decoder_graph(shape, batch=batch, seq=seq, max_len=96, fmt="w8pc", head="argmax", last_token=True)
    logits_id = g.nodes[-1].inputs[0]
    g.outputs.append(logits_id)
    host = seeded_graph_inputs(g, cache_fill=0)
    host[hd.tokens] = ora.uniform_i32(2, batch * seq, 0, shape.vocab)
    host[hd.pos] = np.tile(np.arange(seq, dtype=np.int32), batch)
    res, _ = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in host.items()})
    assert g.values[logits_id].dims == (batch, shape.vocab)
    logits = as_f32(g.values[logits_id], res[logits_id])
    assert_close(logits, ref[logits_id], TOL_BF16, "last-token logits")
    assert np.array_equal(np.asarray(res[hd.out]), ora.argmax(logits))


@pytest.mark.parametrize("batch", [2, 24])
def test_llama70b_gqa_shard_decode(cuda, plugin, batch):
    """70B-shape GQA (64 q / 8 kv heads), one tensor-parallel shard of 8, KV 4096.  Batch 24
    takes the GEMV's two-tiles-per-item path (17-32 x rows) in the q/k/v + RoPE and the
    gate/up + SwiGLU epilogues."""
    g, hd, res, caches, ref = _decode_case(plugin, LLAMA_70B, batch, 1, 4160, 4096, tp_world=8, head="none")
    assert_close(as_f32(g.values[hd.out], res[hd.out]), ref[hd.out], TOL_BF16, "70B shard hidden")


def test_cuda_graph_replay_is_deterministic_and_counted(cuda, plugin):
    g, hd = decoder_graph(LLAMA_7B, batch=2, seq=1, max_len=256, fmt="w4g32", layers=1, head="argmax")
    host = seeded_graph_inputs(g, cache_fill=100)
    host[hd.tokens] = ora.uniform_i32(2, 2, 0, LLAMA_7B.vocab)
    host[hd.pos] = np.full(2, 100, np.int32)
    arena, bufs = {}, []
    for i, v in enumerate(g.values):
        if v.producer is None:
            b = plugin.upload(v.dtype, v.dims, to_device_bytes(v, host[i]))
            bufs.append(b)
            arena[i] = Device(b)
    exe = plugin.compile(g)
    bound = exe.bind(arena)
    outs = []
    for _ in range(4):  # eager, capture, replay, replay
        before = plugin.launch_count()
        bound.run()
        assert plugin.launch_count() > before
        outs.append(bound.outputs[hd.out].read())
    assert all(o == outs[0] for o in outs)
    bound.release()
    for b in bufs:
        b.release()
    exe.free()


def test_bad_token_id_is_an_invalid_argument_not_a_fault(cuda, plugin):
    b = GraphBuilder("emb")
    ids = b.input(I32, (3,), "ids")
    tab = b.input(BF16, (10, 16), "table")
    out = b.node(Op.custom("fused::embed"), [ids, tab], [(BF16, (3, 16))], {}, "embed")[0]
    b.output(out)
    g = b.build()
    with pytest.raises(StrataError) as e:
        run_graph(plugin, g, {ids: np.array([1, 10, 2], np.int32), tab: np.zeros((10, 16), np.float32)})
    assert e.value.code == -3 and "embedding table" in str(e.value)
    # the context stays usable
    res, _ = run_graph(plugin, g, {ids: np.array([1, 9, 2], np.int32), tab: np.ones((10, 16), np.float32)})
    assert np.all(as_f32(g.values[out], res[out]) == 1.0)


def test_device_quantize_node_is_bit_exact(cuda, plugin):
    b = GraphBuilder("quant")
    w = b.input(F32, (64, 256), "w")
    c, s = b.node(Op.custom("fused::quantize_w4g32"), [w], [(W4G32, (64, 128)), (BF16, (64, 8))], {}, "q")
    b.output(c)
    b.output(s)
    g = b.build()
    wv = ora.normal(1, (64, 256), std=0.02)
    res, _ = run_graph(plugin, g, {w: wv})
    want_c, want_s = ora.quant_w4g32(wv)
    assert np.frombuffer(res[c], np.uint8).tobytes() == want_c.tobytes()
    assert np.array_equal(np.asarray(res[s]).view(np.uint16).ravel(), want_s.ravel())


@pytest.mark.parametrize("dtype", [BF16, F32])
@pytest.mark.parametrize("rows,cols,offset", [(1, 4000, 0), (37, 1000, 64000), (300, 16, 31984), (5000, 16, 0)])
def test_vocab_argmax_node_on_one_rank(cuda, plugin, dtype, rows, cols, offset):
    """fused::vocab_argmax outside a tensor-parallel group: the argmax of the
    shard plus its first vocabulary id, with the replicated argmax's rules --
    NaN skipped, the lowest id on ties (-0 and +0 tie), 0 for a row of NaNs.
    5000 rows is more than one peer exchange takes; without an exchange any
    row count is served."""
    b = GraphBuilder("vargmax")
    x = b.input(dtype, (rows, cols), "logits")
    out = b.node(Op.custom("fused::vocab_argmax"), [x], [(I32, (rows,))], {"vocab_offset": offset}, "va")[0]
    b.output(out)
    g = b.build()
    v = ora.normal(3, (rows, cols))
    if dtype == BF16:
        v = ora.round_bf16(v)
    r = np.arange(rows)
    v[r, (r * 7) % cols] = 9.0           # a tie of the row maximum ...
    v[r, (r * 7 + 5) % cols] = 9.0       # ... at a second column
    v[r, (r * 3 + 1) % cols] = np.nan
    v[0, :] = np.where(np.arange(cols) % 2, -0.0, 0.0)  # only zeros of both signs
    if rows > 2:
        v[2, :] = np.nan
        v[1, :] = -np.inf
    res, _ = run_graph(plugin, g, {x: v})
    got = np.asarray(res[out])
    want = ora.argmax(v) + offset
    if rows > 2:
        want[2] = 0
    assert got[0] == offset
    assert np.array_equal(got, want), np.nonzero(got != want)
