"""The drop-in boundary without a GPU: layout, exports, loader sequence,
capabilities, the pull query, compile's tri-state and hostile blobs.

Mirrors the reference's loader/plugin behaviour
(crates/ferrite-strata-plugin-api/src/host/{loader,plugin}.rs) and its wire
tests (crates/ferrite-strata-plugin-api/tests/wire.rs:445-680)."""
import ctypes as C
import os
import re
import struct

import pytest

from strata_host import BF16, F32, I32, W4G32, DType, GraphBuilder, Op, StrataError, w8pc
from strata_host import abi
from strata_host.blocks import BLOCK_512, LLAMA_7B, LLAMA_70B, DecoderShape, decoder_graph
from strata_host.ir import SECTION_GRAPH, encode_graph, frame
from tests.conftest import LIB, ROOT


def test_struct_layouts_match_the_header():
    # The C header pins the same sizes with static_assert (x86-64).
    assert C.sizeof(abi.StrataExtBase) == 24
    assert C.sizeof(abi.StrataPluginVersionExt) == 40
    assert C.sizeof(abi.StrataMessageExt) == 32
    assert C.sizeof(abi.StrataDType) == 16
    assert C.sizeof(abi.StrataShapeClass) == 8
    assert C.sizeof(abi.StrataPatternQuery) == 48
    assert C.sizeof(abi.StrataWireBlob) == 40
    assert C.sizeof(abi.StrataCompileArgs) == 112
    assert C.sizeof(abi.StrataBufferRef) == 16
    assert C.sizeof(abi.StrataRunArgs) == 40
    assert C.sizeof(abi.StrataAllocDesc) == 40
    assert C.sizeof(abi.StrataPluginV1) == 24 + 22 * 8


def test_library_exports_every_declared_symbol(plugin):
    lib = C.CDLL(LIB)
    declared = set()
    for h in ("strata_plugin.h", "strata_b200.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        declared |= set(re.findall(r"\b(strata_b200_\w+)\s*\(", text))
    declared.add("strata_plugin_v1")
    assert len(declared) > 10
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} is declared in include/ but not exported"


def test_vtable_negotiates_and_has_every_mandatory_entry(plugin):
    vt = plugin.vt
    assert vt.struct_size == C.sizeof(abi.StrataPluginV1)
    assert (vt.abi_version.major, vt.abi_version.minor) == (0, 1)
    for name in abi.MANDATORY + ("alloc", "buffer_release", "buffer_write", "buffer_read",
                                 "plugin_init", "plugin_free"):
        assert getattr(vt, name), name
    assert plugin.version == (0, 1, 0, (0, 1))
    assert plugin.device_ext is not None and plugin.device_ext.version == 1


def test_capability_blob(plugin):
    caps = plugin.capabilities
    assert caps.backend_name == "b200"
    assert caps.accepts_unpartitioned
    assert caps.max_rank == 8
    levels = {(p.pattern_id, p.dtype.element): p.level for p in caps.patterns}
    for pid in ("fused::linear_w4g32", "fused::linear_w8pc", "fused::rms_norm", "fused::rope",
                "fused::swiglu", "fused::attention", "fused::embed", "fused::all_reduce"):
        assert levels[(pid, 14)] == abi.SUPPORT_FUSED
    assert levels[("ref::linear", 4)] == abi.SUPPORT_FALLBACK
    # dtype mask bits are ElementType::all() positions: f32, bf16, i8, i32, u8, and the MX
    # formats f8e4m3, f8e8m0, f4e2m1
    assert caps.dtype_mask == ((1 << 3) | (1 << 5) | (1 << 8) | (1 << 10) | (1 << 12) |
                               (1 << 1) | (1 << 6) | (1 << 7))
    for pid in ("fused::linear_mxfp8", "fused::linear_mxfp4"):
        assert levels[(pid, 14)] == abi.SUPPORT_FUSED


ALL_CLASSES = [(), (0, 4), (1, 4096), (64,), (8, 4096), (2, 3, 4), (2, 3, 4, 5), (2,) * 5, (2,) * 8]


@pytest.mark.parametrize("dims", ALL_CLASSES)
def test_pull_query_accepts_every_hot_path_pattern(plugin, dims):
    fused = abi.SUPPORT_FUSED
    assert plugin.supports("fused::linear_w4g32", BF16, dims) == fused
    assert plugin.supports("fused::linear_w8pc", BF16, dims) == fused
    for pid in ("fused::rms_norm", "fused::rope", "fused::swiglu", "fused::attention", "fused::embed"):
        assert plugin.supports(pid, BF16, dims) == fused
        assert plugin.supports(pid, F32, dims) == fused
    assert plugin.supports("fused::argmax", I32, dims) == fused
    assert plugin.supports("fused::vocab_argmax", I32, dims) == fused
    assert plugin.supports("ref::add", BF16, dims) == abi.SUPPORT_FALLBACK
    assert plugin.supports("ref::linear", F32, dims) == abi.SUPPORT_FALLBACK


def test_pull_query_refuses_what_it_cannot_run(plugin):
    assert plugin.supports("fused::flash_attention_v3", BF16, (2, 8)) == abi.SUPPORT_REFUSE
    assert plugin.supports("fused::linear_w4g32", F32, (2, 8)) == abi.SUPPORT_REFUSE
    assert plugin.supports("ref::matmul", BF16, (2, 8)) == abi.SUPPORT_REFUSE
    assert plugin.supports("ref::gelu", DType(3), (2, 8)) == abi.SUPPORT_REFUSE  # f16


@pytest.mark.parametrize("graph_fn", [
    lambda: decoder_graph(BLOCK_512, batch=1, seq=128, max_len=128, fmt="f32", embed=False, head="none")[0],
    lambda: decoder_graph(LLAMA_7B, batch=8, seq=1, max_len=2112, fmt="w4g32")[0],
    lambda: decoder_graph(LLAMA_7B, batch=8, seq=2048, max_len=2048, fmt="w8pc", layers=2)[0],
    lambda: decoder_graph(LLAMA_70B, batch=32, seq=1, max_len=4160, fmt="w4g32", layers=4,
                          tp_rank=3, tp_world=8, head="none")[0],
], ids=["f32_block", "7b_decode", "7b_prefill", "70b_tp8"])
def test_hot_path_graphs_compile_without_decline(plugin, graph_fn):
    exe = plugin.compile(graph_fn())
    assert exe is not None
    exe.free()
    assert plugin.compile(graph_fn(), probe=True) is not None


def _exe_header_offset(payload: bytes) -> int:
    """Offset of the serialised executable's header section in a framed payload."""
    count = struct.unpack_from("<I", payload, 0)[0]
    for i in range(count):
        kind, off, _ = struct.unpack_from("<IQQ", payload, 4 + 20 * i)
        if kind == 0x45583242:
            return off
    raise AssertionError("no executable header section")


@pytest.mark.parametrize("graph_fn", [
    lambda: decoder_graph(LLAMA_7B, batch=2, seq=1, max_len=256, fmt="w4g32", layers=2)[0],
    lambda: decoder_graph(LLAMA_70B, batch=32, seq=1, max_len=4160, fmt="w4g32", layers=1,
                          tp_rank=1, tp_world=8, head="none")[0],
], ids=["7b_decode", "70b_tp8"])
def test_executable_serialises_and_loads_back(plugin, graph_fn):
    """The ahead-of-time entries (raw.rs:760-788): serialize, abi_compatible and
    deserialize_load round-trip an executable with no device work, and the loaded
    executable serialises to the same bytes (same graph, same lowered plan)."""
    g = graph_fn()
    exe = plugin.compile(g)
    blob = plugin.serialize(exe)
    assert plugin.abi_compatible(blob)
    exe2 = plugin.deserialize(blob, g)
    assert exe2.handle and exe2.handle != exe.handle
    assert plugin.serialize(exe2) == blob
    exe.free()
    exe2.free()


def test_foreign_or_tampered_executable_blobs_are_refused(plugin):
    g = decoder_graph(LLAMA_7B, batch=1, seq=1, max_len=128, fmt="w4g32", layers=1)[0]
    exe = plugin.compile(g)
    blob = plugin.serialize(exe)
    exe.free()
    # a subgraph blob is not an executable
    subgraph = frame([(SECTION_GRAPH, encode_graph(g))])[abi.WIRE_HEADER_LEN:]
    assert not plugin.abi_compatible(subgraph)
    with pytest.raises(StrataError) as e:
        plugin.deserialize(subgraph, g)
    assert e.value.code == abi.INVALID_ARGUMENT
    off = _exe_header_offset(blob)
    # another architecture
    other = bytearray(blob)
    struct.pack_into("<I", other, off + 4, 90)
    assert not plugin.abi_compatible(bytes(other))
    # a plan this build does not produce (fingerprint changed): loadable header, refused load
    stale = bytearray(blob)
    struct.pack_into("<Q", stale, off + 16, struct.unpack_from("<Q", blob, off + 16)[0] ^ 1)
    assert plugin.abi_compatible(bytes(stale))
    with pytest.raises(StrataError) as e:
        plugin.deserialize(bytes(stale), g)
    assert e.value.code == abi.INVALID_ARGUMENT
    # truncated
    assert not plugin.abi_compatible(blob[: off + 8])


def _one_node(op, in_dt=F32, out_dt=F32, dims=(1, 4)):
    b = GraphBuilder("g")
    x = b.input(in_dt, dims, "x")
    o = b.node(op, [x], [(out_dt, dims)], {}, "n0")[0]
    b.output(o)
    return b.build()


def test_decline_is_not_an_error(plugin):
    assert plugin.compile(_one_node(Op.custom("fused::flash_attention_v3"))) is None
    b = GraphBuilder("dangling")
    x = b.input(F32, (1, 2), "x")
    b.node(Op("gelu"), [x], [(F32, (1, 2))], {}, "g")
    assert plugin.compile(b.build()) is None  # no outputs
    b = GraphBuilder("bf16mm")
    x = b.input(BF16, (2, 2), "x")
    y = b.input(BF16, (2, 2), "y")
    b.output(b.node(Op("matmul"), [x, y], [(BF16, (2, 2))], {}, "mm")[0])
    assert plugin.compile(b.build()) is None


def test_malformed_graph_is_an_error(plugin):
    b = GraphBuilder("mm")
    x = b.input(F32, (2, 3), "x")
    y = b.input(F32, (2, 2), "y")
    b.output(b.node(Op("matmul"), [x, y], [(F32, (2, 2))], {}, "mm")[0])
    with pytest.raises(StrataError) as e:
        plugin.compile(b.build())
    assert e.value.code == abi.INVALID_ARGUMENT and "inner dimensions" in str(e.value)


def _compile_raw(plugin, payload: bytes, magic=abi.MAGIC, major=abi.FORMAT_MAJOR):
    buf = (C.c_uint8 * max(len(payload), 1)).from_buffer_copy(payload + b"\0")
    args = abi.StrataCompileArgs()
    args.struct_size = C.sizeof(args)
    args.subgraph.magic = magic
    args.subgraph.format_major = major
    args.subgraph.payload_len = len(payload)
    args.subgraph.data = C.cast(buf, C.POINTER(C.c_uint8))
    out, err = C.c_void_p(), C.c_void_p()
    rc = plugin.vt.compile(plugin.ctx, C.byref(args), C.byref(out), C.byref(err))
    msg = ""
    if err.value:
        msg = str(plugin.take_error(err.value, rc))
    if out.value:
        plugin.vt.free_executable(plugin.ctx, out.value)
    return rc, msg


def _payload(section: bytes) -> bytes:
    return frame([(SECTION_GRAPH, section)])[abi.WIRE_HEADER_LEN:]


def _good_section():
    return encode_graph(_one_node(Op("gelu")))


def test_a_well_formed_raw_blob_compiles(plugin):
    assert _compile_raw(plugin, _payload(_good_section()))[0] == abi.OK


@pytest.mark.parametrize("mutate,needle", [
    (lambda s: s[:len(s) // 2], "truncated"),
    (lambda s: s[:4] + struct.pack("<I", 1 << 30) + s[8:], "length overflow"),
    (lambda s: struct.pack("<I", 2) + s[4:], "schema"),
])
def test_hostile_graph_sections_are_rejected(plugin, mutate, needle):
    rc, msg = _compile_raw(plugin, _payload(mutate(_good_section())))
    assert rc == abi.INVALID_ARGUMENT and needle in msg, msg


def test_bad_magic_and_major_are_rejected(plugin):
    assert _compile_raw(plugin, _payload(_good_section()), magic=1)[0] == abi.INVALID_ARGUMENT
    assert _compile_raw(plugin, _payload(_good_section()), major=7)[0] == abi.INVALID_ARGUMENT


def _section_with(values=None, nodes=None, outputs=None):
    """Hand-written graph section (wire/graph.rs:5-29) for the hostile cases."""
    def s(x):
        raw = x.encode()
        return struct.pack("<I", len(raw)) + raw
    out = struct.pack("<I", 1) + s("g")
    values = values or []
    out += struct.pack("<I", len(values))
    for elem, qk, rank, dims, prod, name in values:
        out += struct.pack("<IIIB", elem, qk, 1 if qk else 0, 1 if qk else 0) + struct.pack("<I", rank)
        out += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<QI", prod, 0) + s(name)
    nodes = nodes or []
    out += struct.pack("<I", len(nodes))
    for op, ins, outs, name in nodes:
        out += struct.pack("<I", op) + struct.pack("<I", len(ins)) + b"".join(struct.pack("<I", i) for i in ins)
        out += struct.pack("<I", len(outs)) + b"".join(struct.pack("<I", o) for o in outs)
        out += struct.pack("<I", 0) + s(name)
    outputs = outputs or []
    out += struct.pack("<I", len(outputs)) + b"".join(struct.pack("<I", o) for o in outputs)
    return out


NOP = 0xFFFFFFFFFFFFFFFF


@pytest.mark.parametrize("section,needle", [
    (_section_with([(4, 0, 2, (1, 4), NOP, "x"), (4, 0, 2, (1, 4), (1 << 63) | 0, "y")],
                   [(99, [0], [1], "n")], [1]), "unknown op tag"),
    (_section_with([(4, 0, 2, (1, 4), (1 << 63) | 1, "x"), (4, 0, 2, (1, 4), (1 << 63) | 0, "y")],
                   [(8, [0], [1], "n"), (8, [1], [0], "m")], [1]), "before it is defined"),
    (_section_with([(4, 0, 2, (1, 4), NOP, "x")], [], [0, 0]), "listed twice"),
    (_section_with([(8, 0, 1, (4,), NOP, "ids")], [], [0]), "no scaling convention"),
    (_section_with([(4, 0, 9, (1,) * 9, NOP, "x")], [], [0]), "rank 9"),
    (_section_with([(1, 0, 1, (4,), NOP, "x")], [], [0]), "element-type"),
    (_section_with([(4, 0, 2, (1, 4), NOP, "x"), (4, 0, 2, (1, 4), NOP, "x")], [], [0]), "duplicate name"),
])
def test_hostile_graphs_are_rejected(plugin, section, needle):
    rc, msg = _compile_raw(plugin, _payload(section))
    assert rc == abi.INVALID_ARGUMENT and needle in msg, msg


def test_unknown_sections_are_skipped(plugin):
    payload = frame([(77, b"future section"), (SECTION_GRAPH, _good_section())])[abi.WIRE_HEADER_LEN:]
    assert _compile_raw(plugin, payload)[0] == abi.OK


def test_run_without_a_device_fails_loudly(plugin):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    exe = plugin.compile(_one_node(Op("gelu")))
    with pytest.raises(StrataError) as e:
        exe.run({0: b"\0" * 16})
    assert e.value.code == abi.INTERNAL and "no CUDA device" in str(e.value)
    exe.free()


def test_bare_integer_dtype_is_rejected_by_the_host_builder():
    with pytest.raises(ValueError):
        DType.plain("i32")
    assert W4G32.quant_kind == 1 and w8pc(4096).block_size == 4096


def _plan_steps(plugin, g) -> int:
    """Steps of the lowered plan, read from the serialised executable's header
    (u32 format, u32 arch, u32 abi major, u32 abi minor, u64 fingerprint, u32 steps)."""
    exe = plugin.compile(g)
    assert exe is not None
    blob = plugin.serialize(exe)
    exe.free()
    return struct.unpack_from("<I", blob, _exe_header_offset(blob) + 24)[0]


def test_tensor_parallel_layer_lowers_to_fused_steps(plugin):
    """A tensor-parallel decode layer lowers to 10 steps: embed, RMSNorm, q/k/v GEMV with RoPE
    and cache append, attention, o_proj, all-reduce + residual add + RMSNorm, gate/up GEMV with
    SwiGLU, down_proj, all-reduce + residual add + final RMSNorm, lm_head.  Without the fused
    all-reduce step it would be 14."""
    shape = LLAMA_7B
    for rank in (0, 7):  # 7B FFN shards at 8 ranks: 1408 and 1344 features
        g = decoder_graph(shape, batch=4, seq=1, max_len=256, fmt="w4g32", layers=1, head="logits",
                          tp_rank=rank, tp_world=8)[0]
        assert _plan_steps(plugin, g) == 10
    # the same layer unsharded (10 as well): the residual adds ride on the o_proj and down_proj
    # GEMV epilogues, and the two RMSNorms after them are steps of their own
    g1 = decoder_graph(shape, batch=4, seq=1, max_len=256, fmt="w4g32", layers=1, head="logits")[0]
    assert _plan_steps(plugin, g1) == 10


def test_decode_and_prefill_layers_lower_to_their_fused_plans(plugin):
    """Per-layer plan sizes (one more layer adds exactly these steps): a 7B decode layer is 7
    steps (RMSNorm, q/k/v GEMV with RoPE and cache append, attention, o_proj with residual,
    RMSNorm, gate/up GEMV with SwiGLU, down_proj with residual); an int8 prefill layer is 10
    (q/k/v as one grouped GEMM step, separate RoPE and cache-append steps)."""
    def per_layer(**kw):
        one = _plan_steps(plugin, decoder_graph(LLAMA_7B, layers=1, **kw)[0])
        two = _plan_steps(plugin, decoder_graph(LLAMA_7B, layers=2, **kw)[0])
        return two - one, one
    assert per_layer(batch=2, seq=1, max_len=256, fmt="w4g32", head="argmax") == (7, 11)
    assert per_layer(batch=2, seq=96, max_len=96, fmt="w8pc", head="logits", last_token=True) == (10, 14)
    # paged caches lower to the same plans (the table rides along with the append and attention)
    assert per_layer(batch=2, seq=1, max_len=256, fmt="w4g32", head="argmax", kv_page=16) == (7, 11)
    assert per_layer(batch=2, seq=96, max_len=96, fmt="w8pc", head="logits", last_token=True,
                     kv_page=32) == (10, 14)


@pytest.mark.parametrize("page", [16, 64, 128, 1024])
@pytest.mark.parametrize("seq", [1, 160])
def test_paged_cache_graphs_compile(plugin, page, seq):
    g = decoder_graph(LLAMA_7B, batch=3, seq=seq, max_len=320, fmt="w4g32", layers=1, kv_page=page,
                      kv_pages=2 * 3 * (-(-320 // page)))[0]
    exe = plugin.compile(g)
    assert exe is not None
    exe.free()


def test_paged_cache_rules(plugin):
    """Pages must be a power of two from 16 to 4096 and the pools' third
    dimension; paged f32 caches are declined (the paged kernels are bf16)."""
    small = DecoderShape(256, 4, 2, 64, 512, 0, 1)
    with pytest.raises(StrataError):
        plugin.compile(decoder_graph(small, batch=2, seq=1, max_len=96, fmt="w4g32", embed=False, head="none",
                                     kv_page=48)[0])
    with pytest.raises(StrataError):
        plugin.compile(decoder_graph(small, batch=2, seq=1, max_len=96, fmt="w4g32", embed=False, head="none",
                                     kv_page=8)[0])
    g = decoder_graph(small, batch=2, seq=1, max_len=96, fmt="f32", embed=False, head="none", kv_page=16)[0]
    assert plugin.compile(g) is None


def test_step_times_export_answers_without_a_gpu():
    """strata_b200_step_times: JSON of the per-class totals (none yet: "{}"),
    the bytes needed returned even when the buffer is too small."""
    lib = C.CDLL(LIB)
    fn = lib.strata_b200_step_times
    fn.argtypes = [C.c_char_p, C.c_uint64, C.c_int32]
    fn.restype = C.c_uint64
    need = fn(None, 0, 0)
    buf = C.create_string_buffer(int(need) + 1)
    assert fn(buf, len(buf), 1) == need
    assert buf.value.decode() == "{}"
    small = C.create_string_buffer(1)
    assert fn(small, 1, 0) == need and small.value == b""
