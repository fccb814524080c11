"""Shared helpers for the parity tests: seeded inputs and tolerance checks."""
from __future__ import annotations

import numpy as np

from oracle import oracle as ora
from strata_host import BF16, F32, I32, W4G32
from strata_host.ir import ELEM

# Tolerances from the acceptance bar: max relative error (max |got - want| over
# max |want|) at most 1e-4 for f32 outputs and 2e-2 for bf16 outputs.
TOL_F32 = 1e-4
TOL_BF16 = 2e-2


def max_rel_err(got, want) -> float:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    denom = np.max(np.abs(want))
    return float(np.max(np.abs(got - want)) / (denom if denom > 0 else 1.0))


def assert_close(got, want, tol, what=""):
    err = max_rel_err(got, want)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert err <= tol, f"{what}: max rel err {err:.3e} > {tol:g}"
    return err


def seeded_graph_inputs(graph, seed_base: int = 1, weight_std: float = 0.02,
                        act_seed: int = 0, cache_fill: int | None = None, vocab: int = 0):
    """Host values for every graph input, in declaration order.

    Weights ~ N(0, weight_std) from seed 1 + i (i = input index), quantised by
    the oracle for int4/int8 formats; activations ~ N(0, 1) from seed 0;
    norm gains are 1 + N(0, 0.02); caches ~ N(0, 1) for positions below
    `cache_fill`; ids uniform over the vocabulary from seed 2.
    """
    vals = {}
    for i, v in enumerate(graph.values):
        if v.producer is not None:
            continue
        name = v.name
        seed = seed_base + i
        if v.dtype == I32:
            continue  # ids / positions are set by the caller
        if name in ("x",):
            vals[i] = ora.normal(act_seed, v.dims)
        elif "norm" in name:
            vals[i] = 1.0 + ora.normal(seed, v.dims, std=0.02)
        elif name.endswith("pages"):  # paged cache pools: every page random
            vals[i] = ora.normal(seed, v.dims)
        elif name.endswith("cache"):
            c = np.zeros(v.dims, np.float32)
            if cache_fill:
                c[:, :, :cache_fill, :] = ora.normal(seed, (v.dims[0], v.dims[1], cache_fill, v.dims[3]))
            vals[i] = c
        elif name == "embed_table":
            vals[i] = ora.normal(seed, v.dims)
        elif v.dtype == W4G32:
            n, kh = v.dims
            w = ora.normal(seed, (n, kh * 2), std=weight_std)
            packed, s = ora.quant_w4g32(w)
            vals[i] = packed
            vals[i + 1] = s  # the scale input is declared right after its codes
        elif v.dtype.element in (ELEM["f8e4m3"], ELEM["f4e2m1"]):  # MX codes, then their E8M0 scales
            n, k = v.dims
            w = ora.normal(seed, (n, k), std=weight_std)
            codes, s = ora.quant_mx(w, "mxfp8" if v.dtype.element == ELEM["f8e4m3"] else "mxfp4")
            vals[i] = codes
            vals[i + 1] = s
        elif v.dtype.element == ELEM["i8"]:
            n, k = v.dims
            w = ora.normal(seed, (n, k), std=weight_std)
            q, s = ora.quant_w8pc(w)
            vals[i] = q
            vals[i + 1] = s
        elif i in vals:
            continue  # a scale filled by its codes
        else:
            vals[i] = ora.normal(seed, v.dims, std=weight_std)
        if v.dtype == BF16 and i in vals and vals[i].dtype == np.float32:
            vals[i] = ora.round_bf16(vals[i])
    return vals


def to_device_bytes(v, arr) -> bytes:
    """Host array -> the bytes the graph's dtype declares."""
    if v.dtype == BF16:
        a = np.asarray(arr)
        return (a if a.dtype == np.uint16 else ora.to_bf16(a)).tobytes()
    if v.dtype == F32:
        return np.ascontiguousarray(arr, np.float32).tobytes()
    if v.dtype.element == ELEM["i32"]:
        return np.ascontiguousarray(arr, np.int32).tobytes()
    return np.ascontiguousarray(arr).tobytes()


def page_table(batch: int, pages_per_seq: int, num_pages: int, seed: int = 5) -> np.ndarray:
    """A block table I32 [batch, pages_per_seq] that gives every sequence
    distinct pages of a pool of num_pages, in a seeded random order (pages
    of one sequence are neither consecutive nor ordered)."""
    assert num_pages >= batch * pages_per_seq
    perm = np.random.default_rng(seed).permutation(num_pages)[:batch * pages_per_seq]
    return perm.reshape(batch, pages_per_seq).astype(np.int32)


def to_pages(cache: np.ndarray, table: np.ndarray, num_pages: int, fill_seed: int | None = None) -> np.ndarray:
    """Contiguous caches [B, G, L, d] scattered into a page pool
    [num_pages, G, page, d] through the table (page = L / pages_per_seq).
    Pages no sequence uses hold N(0, 1) noise from fill_seed (zeros if None),
    so a kernel that reads a wrong page shows it."""
    B, G, L, d = cache.shape
    pps = table.shape[1]
    page = L // pps
    pool = np.zeros((num_pages, G, page, d), np.float32)
    if fill_seed is not None:
        pool[:] = ora.normal(fill_seed, pool.shape)
    for b in range(B):
        for lp in range(pps):
            pool[table[b, lp]] = cache[b, :, lp * page:(lp + 1) * page, :]
    return pool


def from_pages(pool: np.ndarray, table: np.ndarray) -> np.ndarray:
    """The contiguous caches [B, G, pages_per_seq * page, d] a pool holds."""
    B, pps = table.shape
    _, G, page, d = pool.shape
    out = np.zeros((B, G, pps * page, d), pool.dtype)
    for b in range(B):
        for lp in range(pps):
            out[b, :, lp * page:(lp + 1) * page, :] = pool[table[b, lp]]
    return out
