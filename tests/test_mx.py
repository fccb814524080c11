"""MX weights (OCP Microscaling: E4M3 or E2M1 codes, one E8M0 scale per 32
along K) behind fused::linear_mxfp8 / fused::linear_mxfp4.

The reference names the element types (crates/ferrite-strata/src/dtype.rs:
41-85, DType::microscaled) but computes none of them, so the oracle's
encodings are pinned here by known values of the formats.  On the GPU the
decode GEMV (codes turned into bf16 in registers) and the prefill GEMM (an
exact bf16 expansion, then the tcgen05 GEMM) are compared with the oracle's
k-order f32 linear within the bf16 tolerance, and codes the formats treat
specially (E4M3 subnormals, both zeros, the largest codes, E8M0 scales near
both ends of the range the kernels take) are exercised directly."""
import numpy as np
import pytest

from oracle import graph_eval, oracle as ora
from strata_host import BF16, E2M1, E4M3, E8M0, GraphBuilder, Op
from strata_host.blocks import DecoderShape, decoder_graph
from tests.helpers import TOL_BF16, assert_close, seeded_graph_inputs

MX_SHAPE = DecoderShape(1024, 8, 8, 128, 2816, 512, 2)


# ---------------------------------------------------------------------------
# oracle known answers (CPU)
# ---------------------------------------------------------------------------
def test_e4m3_known_values_and_round_trip():
    L = ora.lib()
    known = {0x00: 0.0, 0x80: -0.0, 0x01: 2.0 ** -9, 0x07: 7 * 2.0 ** -9, 0x08: 2.0 ** -6, 0x38: 1.0,
             0x3F: 1.875, 0x40: 2.0, 0x7E: 448.0, 0xFE: -448.0, 0xB8: -1.0}
    for c, v in known.items():
        assert L.ora_e4m3_to_f32(c) == v, hex(c)
    assert np.isnan(L.ora_e4m3_to_f32(0x7F)) and np.isnan(L.ora_e4m3_to_f32(0xFF))
    for c in range(256):
        if c & 0x7F != 0x7F:
            assert L.ora_f32_to_e4m3(L.ora_e4m3_to_f32(c)) == c, hex(c)
    # nearest even on ties, saturation at 448
    assert L.ora_f32_to_e4m3(1.0625) == 0x38 and L.ora_f32_to_e4m3(1.1875) == 0x3A
    assert L.ora_f32_to_e4m3(2.0 ** -10) == 0x00 and L.ora_f32_to_e4m3(3 * 2.0 ** -10) == 0x02
    assert L.ora_f32_to_e4m3(470.0) == 0x7E and L.ora_f32_to_e4m3(-1e9) == 0xFE


def test_e2m1_known_values_and_round_trip():
    L = ora.lib()
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for c in range(16):
        v = L.ora_e2m1_to_f32(c)
        assert v == (-1 if c & 8 else 1) * mags[c & 7]
        assert L.ora_f32_to_e2m1(v) == c
    ties = {0.25: 0, 0.75: 2, 1.25: 2, 1.75: 4, 2.5: 4, 3.5: 6, 5.0: 6, 100.0: 7}
    for x, c in ties.items():
        assert L.ora_f32_to_e2m1(x) == c, x


@pytest.mark.parametrize("fmt,emax", [("mxfp8", 8), ("mxfp4", 2)])
def test_mx_quantisation_scales_and_error(fmt, emax):
    """The block scale is 2^(floor(log2 amax) - emax); dequantisation is
    exact (code times a power of two) and within half a code step of the
    weight, except where the largest values saturate."""
    w = ora.normal(3, (16, 256), std=0.02)
    w[0, :32] = 0.0                     # an all-zero block takes scale code 0
    w[1, 32:64] = 2.0 ** np.arange(32) / 2.0 ** 20
    codes, s = ora.quant_mx(w, fmt)
    for r in range(16):
        for b in range(8):
            amax = float(np.max(np.abs(w[r, b * 32:(b + 1) * 32])))
            want = 0 if amax == 0 else int(np.floor(np.log2(amax))) - emax + 127
            assert s[r, b] == want
    d = ora.dequant_mx(codes, s, fmt).astype(np.float64)
    assert np.all(d[0, :32] == 0)
    X = np.repeat(2.0 ** (s.astype(np.float64) - 127), 32, axis=1)
    top, rel, floor = (448.0, 2.0 ** -4, 2.0 ** -10) if fmt == "mxfp8" else (6.0, 0.25, 0.25)
    wa = np.abs(w.astype(np.float64))
    sat = wa >= top * X                  # saturated: the largest code
    assert np.all(np.abs(d[sat]) == top * X[sat])
    err = np.abs(d - w)[~sat]
    assert np.all(err <= np.maximum(rel * wa[~sat], floor * X[~sat]))


def test_mx_decoder_graphs_lower(plugin):
    for fmt in ("mxfp8", "mxfp4"):
        for seq in (1, 96):
            g = decoder_graph(MX_SHAPE, batch=2, seq=seq, max_len=128, fmt=fmt, layers=1)[0]
            exe = plugin.compile(g)
            assert exe is not None
            exe.free()


def test_mx_linear_rules(plugin):
    """K must be a multiple of 128 and N of 16, the scales E8M0; other
    shapes are declined (no kernel takes them), like the int4/int8 rules."""
    def graph(k, n, sdt=E8M0):
        b = GraphBuilder("mx")
        x = b.input(BF16, (4, k), "x")
        w = b.input(E4M3, (n, k), "w")
        sc = b.input(sdt, (n, k // 32), "s")
        y = b.node(Op.custom("fused::linear_mxfp8"), [x, w, sc], [(BF16, (4, n))], {}, "lin")[0]
        b.output(y)
        return b.build()
    assert plugin.compile(graph(256, 64)) is not None
    for bad in (graph(96, 64), graph(256, 24), graph(256, 64, BF16)):
        assert plugin.compile(bad) is None


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _mx_linear(fmt, m, n, k):
    b = GraphBuilder("mxlin")
    x = b.input(BF16, (m, k), "x")
    w = b.input(E4M3 if fmt == "mxfp8" else E2M1, (n, k), "w")
    sc = b.input(E8M0, (n, k // 32), "s")
    y = b.node(Op.custom(f"fused::linear_{fmt}"), [x, w, sc], [(BF16, (m, n))], {}, "lin")[0]
    b.output(y)
    return b.build(), x, w, sc, y


def _run_linear(plugin, fmt, m, n, k, codes, scales, xv):
    from tests.test_gpu_plugin import as_f32, run_graph
    g, x, w, sc, y = _mx_linear(fmt, m, n, k)
    res, _ = run_graph(plugin, g, {x: xv, w: codes, sc: scales})
    got = as_f32(g.values[y], res[y])
    want = ora.linear_mx(xv, codes, scales, fmt, threads=ora.max_threads())
    return got, want


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("m", [1, 8, 16, 33, 64, 128, 300])
def test_mx_linear_matches_oracle(cuda, plugin, fmt, m):
    """Decode rows (GEMV, 1-64 rows: 1, 2, 4 and 8 n-tiles) and prefill rows
    (the bf16 expansion and the tcgen05 GEMM) on a 4096 x 4096 layer."""
    n = k = 4096
    codes, s = ora.quant_mx(ora.normal(1, (n, k), std=0.02), fmt)
    xv = ora.round_bf16(ora.normal(0, (m, k)))
    got, want = _run_linear(plugin, fmt, m, n, k, codes, s, xv)
    assert_close(got, want, TOL_BF16, f"{fmt} m={m}")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("m", [4, 96])
def test_mx_every_code_and_extreme_scales(cuda, plugin, fmt, m):
    """Rows of every code (E4M3: all 254 finite codes, subnormals included;
    E2M1: all 16) under block scales from 2^-100 to 2^100, with each row's
    scales varying by block: each output element is compared with the oracle
    relative to its own magnitude (a flushed subnormal or a mis-scaled block
    would show)."""
    n, k = 64, 1024
    rng = np.random.default_rng(7)
    if fmt == "mxfp8":
        finite = np.array([c for c in range(256) if c & 0x7F != 0x7F], np.uint8)
        codes = finite[rng.integers(0, len(finite), (n, k))].astype(np.uint8)
        codes[0, :] = np.resize(np.array([1, 2, 3, 4, 5, 6, 7, 0x81, 0x82, 0x87], np.uint8), k)  # subnormals only
    else:
        nib = rng.integers(0, 16, (n, k)).astype(np.uint8)
        codes = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    s = rng.integers(27, 228, (n, k // 32)).astype(np.uint8)
    s[1, :] = 27
    s[2, :] = 227
    xv = ora.round_bf16(ora.normal(0, (m, k)))
    got, want = _run_linear(plugin, fmt, m, n, k, codes, s, xv)
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
    assert np.all(np.isfinite(got))
    # bf16 output rounding (2^-8) plus f32 accumulation order, against each element's own size,
    # where the element is not a cancellation (tiny against its row)
    big = np.abs(want) > 1e-3 * np.max(np.abs(want), axis=1, keepdims=True)
    assert np.max(rel[big]) < 2 ** -7, float(np.max(rel[big]))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("batch,seq", [(4, 1), (2, 96)])
def test_mx_decoder_step_matches_oracle(cuda, plugin, fmt, batch, seq):
    """Two layers with MX weights everywhere (lm_head included): the decode
    step (fused q/k/v + RoPE + append, SwiGLU, residual epilogues on the MX
    GEMV) and a prefill step (the GEMM path), against the oracle."""
    from tests.test_gpu_plugin import as_f32, run_graph
    fill = 100 if seq == 1 else 0
    g, hd = decoder_graph(MX_SHAPE, batch=batch, seq=seq, max_len=128, fmt=fmt, head="logits")
    host = seeded_graph_inputs(g, cache_fill=fill)
    host[hd.tokens] = ora.uniform_i32(2, batch * seq, 0, MX_SHAPE.vocab)
    host[hd.pos] = (np.array([fill - i for i in range(batch)], np.int32) if seq == 1
                    else np.tile(np.arange(seq, dtype=np.int32), batch))
    res, _ = run_graph(plugin, g, host)
    ref = graph_eval.evaluate(g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in host.items()})
    assert_close(as_f32(g.values[hd.out], res[hd.out]), ref[hd.out], TOL_BF16, f"{fmt} logits")


def _grid(fmt):
    """Every finite value of the element format, with its code, by the
    format's definition (independent of the oracle's arithmetic)."""
    vals = []
    if fmt == "mxfp8":
        for c in range(256):
            e, m = (c >> 3) & 15, c & 7
            if (c & 0x7F) == 0x7F:
                continue
            v = m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7)
            vals.append((-v if c & 0x80 else v, c))
    else:
        for c in range(16):
            e, m = (c >> 1) & 3, c & 1
            v = m * 0.5 if e == 0 else (1 + m / 2) * 2.0 ** (e - 1)
            vals.append((-v if c & 8 else v, c))
    return vals


def _encode_by_search(x, fmt):
    """Nearest representable value, ties to the even code (even mantissa),
    saturating at the largest finite magnitude; zero keeps the sign."""
    grid = _grid(fmt)
    top = max(abs(v) for v, _ in grid)
    sign_bit = 0x80 if fmt == "mxfp8" else 8
    if abs(x) >= top:
        return max((c for v, c in grid if abs(v) == top and (v < 0) == (x < 0)))
    best = min(abs(v - x) for v, _ in grid)
    cands = [(v, c) for v, c in grid if abs(v - x) == best]
    if len(cands) > 1:  # a tie: the even mantissa
        cands = [(v, c) for v, c in cands if (c & 1) == 0] or cands
    v, c = cands[0]
    if v == 0:  # both zeros are nearest: keep x's sign
        c = (sign_bit if np.signbit(x) else 0)
    return c


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
def test_mx_encoders_agree_with_an_independent_search(fmt):
    """The oracle's E4M3 / E2M1 encoders against a nearest-value search over
    every representable value: random magnitudes across the formats' range,
    exact ties and saturation."""
    L = ora.lib()
    enc = L.ora_f32_to_e4m3 if fmt == "mxfp8" else L.ora_f32_to_e2m1
    rng = np.random.default_rng(11)
    top = 448.0 if fmt == "mxfp8" else 6.0
    xs = list((rng.standard_normal(3000) * np.exp(rng.uniform(-12, 6, 3000))).astype(np.float32))
    grid = sorted(v for v, _ in _grid(fmt) if v >= 0)
    xs += [np.float32((a + b) / 2) for a, b in zip(grid, grid[1:])]  # exact midpoints
    xs += [np.float32(-x) for x in xs[-20:]] + [np.float32(top * 1.1), np.float32(-top * 3), np.float32(0.0)]
    for x in xs:
        assert enc(float(x)) == _encode_by_search(float(x), fmt), (fmt, float(x))
