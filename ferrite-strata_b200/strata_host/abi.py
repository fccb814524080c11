"""ctypes mirror of include/strata_plugin.h and include/strata_b200.h.

The field order of every struct follows the reference's
crates/ferrite-strata-plugin-api/src/raw.rs (lines 37-789); the sizes are
pinned by tests/test_abi.py against the C header's static_asserts.
"""
from __future__ import annotations

import ctypes as C

# ---- constants (raw.rs, status.rs) -------------------------------------
ABI_MAJOR, ABI_MINOR = 0, 1
EXT_NONE, EXT_PLUGIN_VERSION, EXT_MESSAGE = 0, 1, 2
EXT_B200_DEVICE = 0x56443242
MAGIC = int.from_bytes(b"STRATAG1", "little")
WIRE_HEADER_LEN = 24
FORMAT_MAJOR, FORMAT_MINOR = 0, 1
ENTRY_SYMBOL = "strata_plugin_v1"

OK, DECLINED = 0, 1
UNIMPLEMENTED, INVALID_ARGUMENT, NOT_FOUND, RESOURCE_EXHAUSTED, INTERNAL = -2, -3, -4, -5, -6
STATUS_NAMES = {
    OK: "ok", DECLINED: "declined", UNIMPLEMENTED: "unimplemented",
    INVALID_ARGUMENT: "invalid-argument", NOT_FOUND: "not-found",
    RESOURCE_EXHAUSTED: "resource-exhausted", INTERNAL: "internal",
}

SUPPORT_REFUSE, SUPPORT_FALLBACK, SUPPORT_FUSED = 0, 1, 2


class StrataAbiVersion(C.Structure):
    _fields_ = [("major", C.c_uint32), ("minor", C.c_uint32)]


class StrataExtBase(C.Structure):
    pass


StrataExtBase._fields_ = [("struct_size", C.c_size_t), ("ty", C.c_uint32),
                          ("next", C.POINTER(StrataExtBase))]


class StrataPluginVersionExt(C.Structure):
    _fields_ = [("base", StrataExtBase), ("major", C.c_uint16), ("minor", C.c_uint16),
                ("patch", C.c_uint16), ("targets", StrataAbiVersion)]


class StrataMessageExt(C.Structure):
    _fields_ = [("base", StrataExtBase), ("message", C.c_char_p)]


class StrataQuantSpec(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("block_size", C.c_uint32), ("symmetric", C.c_uint8)]


class StrataDType(C.Structure):
    _fields_ = [("element", C.c_uint32), ("quant", StrataQuantSpec)]


class StrataShapeClass(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("rank", C.c_uint8), ("reserved", C.c_uint8 * 2)]


class StrataPatternQuery(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("pattern_id", C.c_char_p),
                ("pattern_id_len", C.c_size_t), ("dtype", StrataDType),
                ("shape_class", StrataShapeClass)]


class StrataWireBlob(C.Structure):
    _fields_ = [("magic", C.c_uint64), ("format_major", C.c_uint32),
                ("format_minor", C.c_uint32), ("payload_len", C.c_uint64),
                ("data", C.POINTER(C.c_uint8)), ("nul", C.c_uint8)]


class StrataCompileArgs(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("subgraph", StrataWireBlob),
                ("pattern_id", C.c_char_p), ("pattern_id_len", C.c_size_t),
                ("capabilities", StrataWireBlob), ("probe", C.c_uint8),
                ("reserved", C.c_uint8 * 7)]


class StrataBufferRef(C.Structure):
    _fields_ = [("buffer", C.c_void_p), ("value_index", C.c_uint32), ("reserved", C.c_uint32)]


class StrataArenaEntryView(C.Structure):
    _fields_ = [("element_count", C.c_uint64), ("dtype", StrataDType),
                ("data", C.POINTER(C.c_uint8))]


class StrataArenaView(C.Structure):
    _fields_ = [("entry_count", C.c_uint32), ("entries", C.POINTER(StrataArenaEntryView))]


class StrataRunArgs(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("executable", C.c_void_p),
                ("arg_count", C.c_uint32), ("args", C.POINTER(StrataBufferRef)),
                ("host_arena", C.POINTER(StrataArenaView))]


class StrataAllocDesc(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("dtype", StrataDType), ("rank", C.c_uint32),
                ("reserved", C.c_uint32), ("dims", C.POINTER(C.c_uint64))]


PayloadVisitor = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.POINTER(StrataExtBase))

_vp = C.c_void_p
_FN = C.CFUNCTYPE


class StrataPluginV1(C.Structure):
    _fields_ = [
        ("struct_size", C.c_size_t),
        ("extension_start", C.POINTER(StrataExtBase)),
        ("abi_version", StrataAbiVersion),
        ("error_free", _FN(None, _vp)),
        ("error_code", _FN(C.c_uint32, _vp)),
        ("error_payload", _FN(None, _vp, PayloadVisitor, _vp)),
        ("capabilities", _FN(C.c_int32, _vp, C.POINTER(StrataWireBlob))),
        ("supports", _FN(C.c_uint32, _vp, C.POINTER(StrataPatternQuery))),
        ("compile", _FN(C.c_int32, _vp, C.POINTER(StrataCompileArgs), C.POINTER(_vp), C.POINTER(_vp))),
        ("alloc", _FN(C.c_int32, _vp, C.POINTER(StrataAllocDesc), C.POINTER(_vp), C.POINTER(_vp))),
        ("buffer_release", _FN(C.c_int32, _vp, _vp)),
        ("buffer_write", _FN(C.c_int32, _vp, _vp, C.c_uint64, _vp, C.c_uint64)),
        ("buffer_read", _FN(C.c_int32, _vp, _vp, C.c_uint64, _vp, C.c_uint64)),
        ("buffer_event", _FN(C.c_int32, _vp, _vp, C.POINTER(_vp))),
        ("event_ready", _FN(C.c_int32, _vp, _vp)),
        ("event_await", _FN(C.c_int32, _vp, _vp)),
        ("event_free", _FN(C.c_int32, _vp, _vp)),
        ("run", _FN(C.c_int32, _vp, C.POINTER(StrataRunArgs), C.POINTER(_vp))),
        ("free_executable", _FN(None, _vp, _vp)),
        ("free_blob", _FN(None, _vp, C.POINTER(StrataWireBlob))),
        ("plugin_init", _FN(_vp)),
        ("plugin_free", _FN(None, _vp)),
        ("serialize", _FN(C.c_int32, _vp, _vp, C.POINTER(StrataWireBlob))),
        ("deserialize_load", _FN(C.c_int32, _vp, C.POINTER(StrataWireBlob), C.POINTER(_vp))),
        ("abi_compatible", _FN(C.c_int32, _vp, C.POINTER(StrataWireBlob))),
    ]


MANDATORY = ("error_free", "error_code", "error_payload", "capabilities", "supports",
             "compile", "run", "free_executable", "free_blob")


class StrataB200DeviceExt(C.Structure):
    _fields_ = [
        ("base", StrataExtBase),
        ("version", C.c_uint32),
        ("reserved", C.c_uint32),
        ("buffer_wrap", _FN(C.c_int32, _vp, _vp, C.c_uint64, C.POINTER(_vp))),
        ("buffer_device_ptr", _FN(C.c_int32, _vp, _vp, C.POINTER(_vp), C.POINTER(C.c_uint64))),
        ("run_async", _FN(C.c_int32, _vp, C.POINTER(StrataRunArgs), C.POINTER(_vp))),
        ("synchronize", _FN(C.c_int32, _vp, C.POINTER(_vp))),
        ("stream", _FN(_vp, _vp)),
        ("launch_count", _FN(C.c_uint64, _vp)),
        ("tp_unique_id", _FN(C.c_int32, _vp, C.POINTER(C.c_uint8))),
        ("tp_init", _FN(C.c_int32, _vp, C.c_int32, C.c_int32, C.POINTER(C.c_uint8), C.POINTER(_vp))),
        ("set_device", _FN(C.c_int32, _vp, C.c_int32)),
    ]
