"""Kernel-level parity on the B200, through the C entry points of
include/strata_b200.h (plain device pointers, torch only for memory)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as ora
from tests.helpers import TOL_BF16, assert_close
from tests.conftest import LIB

pytestmark = pytest.mark.gpu

P, I64, F = C.c_void_p, C.c_int64, C.c_float


@pytest.fixture(scope="module")
def lib(cuda):
    lib = C.CDLL(LIB)
    sig = {
        "strata_b200_quant_w4g32": [P, I64, I64, P, P, P],
        "strata_b200_quant_w8pc": [P, I64, I64, P, P, P],
        "strata_b200_dequant_w4g32": [P, P, I64, I64, P, P],
        "strata_b200_dequant_w8pc": [P, P, I64, I64, P, P],
        "strata_b200_linear_w4g32": [P, I64, I64, P, P, I64, P, P, P],
        "strata_b200_linear_w8pc": [P, I64, I64, P, P, I64, P, P, P],
        "strata_b200_linear_mxfp8": [P, I64, I64, P, P, I64, P, P, P],
        "strata_b200_linear_mxfp4": [P, I64, I64, P, P, I64, P, P, P],
        "strata_b200_linear_bf16": [P, I64, I64, P, I64, P, P, P],
        "strata_b200_rms_norm_bf16": [P, P, I64, I64, F, P, P],
        "strata_b200_rope_bf16": [P, P, I64, I64, I64, F, P, P],
        "strata_b200_swiglu_bf16": [P, P, I64, P, P],
        "strata_b200_attention_decode_bf16": [P, P, P, P, P, P, I64, I64, I64, I64, I64, P, P, P],
        "strata_b200_embed_bf16": [P, I64, P, I64, I64, P, P],
        "strata_b200_argmax_bf16": [P, I64, I64, P, P],
    }
    for name, args in sig.items():
        getattr(lib, name).argtypes = args
        getattr(lib, name).restype = C.c_int32
    lib.strata_b200_attention_decode_scratch_bytes.argtypes = [I64, I64, I64, I64]
    lib.strata_b200_attention_decode_scratch_bytes.restype = C.c_uint64
    return lib


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def stream(torch):
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def ok(rc):
    assert rc == 0, f"kernel entry point returned {rc}"


@pytest.mark.parametrize("n,k", [(4096, 4096), (7, 96), (1, 32)])
def test_quant_w4g32_is_bit_exact(cuda, lib, n, k):
    torch = cuda
    w = ora.normal(1, (n, k), std=0.02)
    w[0, :32] = 0.0                 # an all-zero group
    w[-1, -1] = 3.0                 # an outlier
    want_p, want_s = ora.quant_w4g32(w)
    wd = dev(torch, w)
    p = torch.empty((n, k // 2), dtype=torch.uint8, device="cuda")
    s = torch.empty((n, k // 32), dtype=torch.int16, device="cuda")
    ok(lib.strata_b200_quant_w4g32(ptr(wd), n, k, ptr(p), ptr(s), stream(torch)))
    torch.cuda.synchronize()
    assert np.array_equal(p.cpu().numpy(), want_p)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), want_s)
    deq = torch.empty((n, k), dtype=torch.float32, device="cuda")
    ok(lib.strata_b200_dequant_w4g32(ptr(p), ptr(s), n, k, ptr(deq), stream(torch)))
    torch.cuda.synchronize()
    assert np.array_equal(deq.cpu().numpy(), ora.dequant_w4g32(want_p, want_s))


def test_quant_w8pc_is_bit_exact(cuda, lib):
    torch = cuda
    n, k = 1024, 4096
    w = ora.normal(3, (n, k), std=0.02)
    w[5] = 0.0
    want_q, want_s = ora.quant_w8pc(w)
    wd = dev(torch, w)
    q = torch.empty((n, k), dtype=torch.int8, device="cuda")
    s = torch.empty((n,), dtype=torch.float32, device="cuda")
    ok(lib.strata_b200_quant_w8pc(ptr(wd), n, k, ptr(q), ptr(s), stream(torch)))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert np.array_equal(s.cpu().numpy(), want_s)
    deq = torch.empty((n, k), dtype=torch.float32, device="cuda")
    ok(lib.strata_b200_dequant_w8pc(ptr(q), ptr(s), n, k, ptr(deq), stream(torch)))
    torch.cuda.synchronize()
    assert np.array_equal(deq.cpu().numpy(), ora.dequant_w8pc(want_q, want_s))


def _x_bf16(m, k, seed=0):
    return ora.to_bf16(ora.normal(seed, (m, k)))


@pytest.mark.parametrize("m", [1, 2, 3, 8, 16, 32, 128, 2048])
def test_linear_w4g32_matches_oracle(cuda, lib, m):
    """The quantized Linear sweep at K = N = 4096 (int4 group 32, bf16 scale)."""
    torch = cuda
    k = n = 4096
    x = _x_bf16(m, k)
    w = ora.normal(1, (n, k), std=0.02)
    packed, s = ora.quant_w4g32(w)
    xd, pd, sd = dev(torch, x.view(np.int16)), dev(torch, packed), dev(torch, s.view(np.int16))
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    ok(lib.strata_b200_linear_w4g32(ptr(xd), m, k, ptr(pd), ptr(sd), n, None, ptr(y), stream(torch)))
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    rows = np.arange(m) if m <= 128 else np.linspace(0, m - 1, 48).astype(int)
    want = ora.round_bf16(ora.linear_w4g32(ora.from_bf16(x[rows]), packed, s, threads=ora.max_threads()))
    assert_close(got[rows], want, TOL_BF16, f"w4g32 m={m}")


@pytest.mark.parametrize("fmt", ["w4g32", "w8pc"])
@pytest.mark.parametrize("m", [1, 5, 24, 64, 65])
@pytest.mark.parametrize("n,k", [(256, 11008), (48, 2752), (16, 96), (32, 4128), (64, 1376)])
def test_linear_ragged_shapes(cuda, lib, fmt, m, n, k):
    """K-slices that end in partial chunks, odd group counts (K = 96, 4128, and 1376 = the
    7B down_proj at 8-way tensor parallelism) or empty slices, and 1..9 n-tiles of x rows."""
    torch = cuda
    x = _x_bf16(m, k, seed=3)  # odd int4 group counts take the CUDA-core GEMV
    w = ora.normal(4, (n, k), std=0.02)
    xd = dev(torch, x.view(np.int16))
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    if fmt == "w4g32":
        packed, s = ora.quant_w4g32(w)
        pd, sd = dev(torch, packed), dev(torch, s.view(np.int16))
        ok(lib.strata_b200_linear_w4g32(ptr(xd), m, k, ptr(pd), ptr(sd), n, None, ptr(y), stream(torch)))
        want = ora.linear_w4g32(ora.from_bf16(x), packed, s, threads=ora.max_threads())
    else:
        q, s = ora.quant_w8pc(w)
        qd, sd = dev(torch, q), dev(torch, s)
        ok(lib.strata_b200_linear_w8pc(ptr(xd), m, k, ptr(qd), ptr(sd), n, None, ptr(y), stream(torch)))
        want = ora.linear_w8pc(ora.from_bf16(x), q, s, threads=ora.max_threads())
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    assert_close(got, ora.round_bf16(want), TOL_BF16, f"{fmt} m={m} n={n} k={k}")


@pytest.mark.parametrize("m,n,k", [(65, 256, 64), (128, 4096, 4096), (1000, 300, 136), (2048, 512, 4096),
                                   (300, 2560, 1000)])
@pytest.mark.parametrize("residual", [False, True])
def test_linear_bf16_tensor_core_gemm(cuda, lib, m, n, k, residual):
    """More than 64 rows: the tcgen05 GEMM (ragged M, N and K tails, residual epilogue),
    against a float64 product of the same bf16 inputs."""
    torch = cuda
    x = ora.to_bf16(ora.normal(31, (m, k)))
    w = ora.to_bf16(ora.normal(32, (n, k), std=0.05))
    r = ora.to_bf16(ora.normal(33, (m, n))) if residual else None
    xd, wd = dev(torch, x.view(np.int16)), dev(torch, w.view(np.int16))
    rd = dev(torch, r.view(np.int16)) if residual else None
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    ok(lib.strata_b200_linear_bf16(ptr(xd), m, k, ptr(wd), n, ptr(rd), ptr(y), stream(torch)))
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    want = ora.from_bf16(x).astype(np.float64) @ ora.from_bf16(w).astype(np.float64).T
    if residual:
        want = ora.round_bf16(want.astype(np.float32)) + ora.from_bf16(r)
    assert_close(got, ora.round_bf16(np.asarray(want, np.float32)), TOL_BF16, f"bf16 gemm m={m} n={n} k={k}")


@pytest.mark.parametrize("m", [1, 16, 128])
def test_linear_w8pc_matches_oracle(cuda, lib, m):
    torch = cuda
    k = n = 4096
    x = _x_bf16(m, k)
    q, s = ora.quant_w8pc(ora.normal(1, (n, k), std=0.02))
    xd, qd, sd = dev(torch, x.view(np.int16)), dev(torch, q), dev(torch, s)
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    ok(lib.strata_b200_linear_w8pc(ptr(xd), m, k, ptr(qd), ptr(sd), n, None, ptr(y), stream(torch)))
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    want = ora.round_bf16(ora.linear_w8pc(ora.from_bf16(x), q, s, threads=ora.max_threads()))
    assert_close(got, want, TOL_BF16, f"w8pc m={m}")


def test_linear_residual_epilogue(cuda, lib):
    torch = cuda
    m, k, n = 4, 1024, 512
    x = _x_bf16(m, k)
    r = ora.to_bf16(ora.normal(9, (m, n)))
    packed, s = ora.quant_w4g32(ora.normal(1, (n, k), std=0.02))
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    args = [dev(torch, a) for a in (x.view(np.int16), packed, s.view(np.int16), r.view(np.int16))]
    ok(lib.strata_b200_linear_w4g32(ptr(args[0]), m, k, ptr(args[1]), ptr(args[2]), n, ptr(args[3]),
                                    ptr(y), stream(torch)))
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    want = ora.round_bf16(ora.round_bf16(ora.linear_w4g32(ora.from_bf16(x), packed, s)) + ora.from_bf16(r))
    assert_close(got, want, TOL_BF16, "residual epilogue")


def test_rms_norm_rope_swiglu(cuda, lib):
    torch = cuda
    rows, cols = 8, 4096
    x = ora.to_bf16(ora.normal(0, (rows, cols)))
    g = ora.to_bf16(1 + ora.normal(4, (cols,), std=0.02))
    y = torch.empty((rows, cols), dtype=torch.int16, device="cuda")
    xd, gd = dev(torch, x.view(np.int16)), dev(torch, g.view(np.int16))
    ok(lib.strata_b200_rms_norm_bf16(ptr(xd), ptr(gd), rows, cols, 1e-5, ptr(y), stream(torch)))
    pos = np.array([0, 1, 5, 100, 2047, 2048, 4000, 7], np.int32)
    yr = torch.empty((rows, cols), dtype=torch.int16, device="cuda")
    posd = dev(torch, pos)  # device tensors stay referenced until the kernels have run
    ok(lib.strata_b200_rope_bf16(ptr(xd), ptr(posd), rows, 32, 128, 10000.0, ptr(yr), stream(torch)))
    u = ora.to_bf16(ora.normal(6, (rows, cols)))
    ys = torch.empty((rows, cols), dtype=torch.int16, device="cuda")
    ud = dev(torch, u.view(np.int16))
    ok(lib.strata_b200_swiglu_bf16(ptr(xd), ptr(ud), rows * cols, ptr(ys), stream(torch)))
    torch.cuda.synchronize()
    xf, gf, uf = ora.from_bf16(x), ora.from_bf16(g), ora.from_bf16(u)
    assert_close(ora.from_bf16(y.cpu().numpy().view(np.uint16)), ora.round_bf16(ora.rms_norm(xf, gf)), TOL_BF16, "rms")
    assert_close(ora.from_bf16(yr.cpu().numpy().view(np.uint16)), ora.round_bf16(ora.rope(xf, pos, 128)), TOL_BF16, "rope")
    assert_close(ora.from_bf16(ys.cpu().numpy().view(np.uint16)), ora.round_bf16(ora.swiglu(xf, uf)), TOL_BF16, "swiglu")


@pytest.mark.parametrize("batch,heads,kv_heads,max_len,fill,d", [
    (1, 32, 32, 2112, 2048, 128),   # 7B decode, KV 2048 prefilled
    (4, 32, 32, 2112, 2048, 128),
    (2, 64, 8, 4160, 4096, 128),    # 70B GQA, KV 4096
    (3, 8, 2, 300, 17, 128),        # ragged short caches
    (1, 8, 2, 16, 0, 128),          # the first token: position 0, cache of one slab
    (5, 16, 4, 530, 515, 64),       # head_dim 64, 4 query heads per kv head
    (2, 8, 8, 40, 33, 64),          # positions ending inside a 16-position slab
])
def test_attention_decode_matches_oracle(cuda, lib, batch, heads, kv_heads, max_len, fill, d):
    torch = cuda
    kc = np.zeros((batch, kv_heads, max_len, d), np.float32)
    kc[:, :, :fill] = ora.normal(11, (batch, kv_heads, fill, d))
    vc = np.zeros_like(kc)
    vc[:, :, :fill] = ora.normal(12, (batch, kv_heads, fill, d))
    kc, vc = ora.round_bf16(kc), ora.round_bf16(vc)
    q = ora.round_bf16(ora.normal(13, (batch, heads * d)))
    kn = ora.round_bf16(ora.normal(14, (batch, kv_heads * d)))
    vn = ora.round_bf16(ora.normal(15, (batch, kv_heads * d)))
    pos = np.array([fill - b for b in range(batch)], np.int32)  # ragged lengths
    kcd, vcd = dev(torch, ora.to_bf16(kc).view(np.int16)), dev(torch, ora.to_bf16(vc).view(np.int16))
    qd, knd, vnd = (dev(torch, ora.to_bf16(a).view(np.int16)) for a in (q, kn, vn))
    posd = dev(torch, pos)
    scratch_bytes = lib.strata_b200_attention_decode_scratch_bytes(batch, heads, d, max_len)
    scratch = torch.empty((max(scratch_bytes, 4),), dtype=torch.uint8, device="cuda")
    out = torch.empty((batch, heads * d), dtype=torch.int16, device="cuda")
    ok(lib.strata_b200_attention_decode_bf16(ptr(qd), ptr(knd), ptr(vnd), ptr(kcd), ptr(vcd),
                                             ptr(posd), batch, heads, kv_heads, d, max_len,
                                             ptr(scratch), ptr(out), stream(torch)))
    torch.cuda.synchronize()
    for b in range(batch):
        kc[b, :, pos[b]] = kn[b].reshape(kv_heads, d)
        vc[b, :, pos[b]] = vn[b].reshape(kv_heads, d)
    # the kernel appended the new rows into the device caches
    assert np.array_equal(ora.from_bf16(kcd.cpu().numpy().view(np.uint16)), kc)
    want = ora.round_bf16(ora.attention(q, kc, vc, np.arange(batch), pos, heads, kv_heads, d,
                                        threads=ora.max_threads()))
    got = ora.from_bf16(out.cpu().numpy().view(np.uint16))
    assert_close(got, want, TOL_BF16, "attention")


def test_embed_and_argmax_are_exact(cuda, lib):
    torch = cuda
    vocab, dim, rows = 32000, 4096, 8
    table = ora.to_bf16(ora.normal(21, (vocab, dim)))
    ids = ora.uniform_i32(2, rows, 0, vocab)
    out = torch.empty((rows, dim), dtype=torch.int16, device="cuda")
    idsd, tabd = dev(torch, ids), dev(torch, table.view(np.int16))
    ok(lib.strata_b200_embed_bf16(ptr(idsd), rows, ptr(tabd), vocab,
                                  dim, ptr(out), stream(torch)))
    logits = ora.to_bf16(ora.normal(22, (rows, vocab)))
    logits[0, 5] = logits[0, 900] = 0x4200  # tie at the maximum (32.0): lowest index wins
    logits[1, :] = 0x7FC0                   # all NaN
    logits[1, 77] = 0x3F80
    am = torch.empty((rows,), dtype=torch.int32, device="cuda")
    lgd = dev(torch, logits.view(np.int16))
    ok(lib.strata_b200_argmax_bf16(ptr(lgd), rows, vocab, ptr(am), stream(torch)))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), table[ids])
    got = am.cpu().numpy()
    assert np.array_equal(got, ora.argmax(ora.from_bf16(logits)))
    assert got[0] == 5 and got[1] == 77


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (24, 256, 11008), (64, 48, 384), (200, 512, 1024)])
def test_linear_mx_entry_points(cuda, lib, fmt, m, n, k):
    """strata_b200_linear_mxfp8 / _mxfp4 with a residual: the GEMV (K-slices
    of 11008 = 86 four-group blocks, partial chunks at K = 384) and, past 64
    rows, the exact bf16 expansion and the tcgen05 GEMM."""
    torch = cuda
    x = _x_bf16(m, k, seed=6)
    codes, s = ora.quant_mx(ora.normal(8, (n, k), std=0.02), fmt)
    res = ora.to_bf16(ora.normal(9, (m, n)))
    xd, cd, sd = dev(torch, x.view(np.int16)), dev(torch, codes), dev(torch, s)
    rd = dev(torch, res.view(np.int16))
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    fn = lib.strata_b200_linear_mxfp8 if fmt == "mxfp8" else lib.strata_b200_linear_mxfp4
    ok(fn(ptr(xd), m, k, ptr(cd), ptr(sd), n, ptr(rd), ptr(y), stream(torch)))
    torch.cuda.synchronize()
    got = ora.from_bf16(y.cpu().numpy().view(np.uint16))
    want = ora.linear_mx(ora.from_bf16(x), codes, s, fmt, threads=ora.max_threads()) + ora.from_bf16(res)
    assert_close(got, want, TOL_BF16, f"{fmt} m={m} n={n} k={k}")
