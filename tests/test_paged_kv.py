"""Paged KV caches (block tables): each layer's k/v caches are page pools and
one block table maps every sequence's positions to pages.

On the CPU the oracle's paged attention must equal its contiguous attention
exactly.  On the GPU the paged step must equal the contiguous step bit for
bit: it runs the same kernels with the same splits and only the cache
addressing differs.  That holds for decode (the q/k/v GEMV appends through
the table, the decode attention reads slabs through it) and prefill (the
append kernel, the tcgen05 attention's TMA loads page by page).  The pool
pages no sequence uses hold noise, so a read of a wrong page would show."""
import numpy as np
import pytest

from oracle import graph_eval, oracle as ora
from strata_host import BF16, Device, StrataError
from strata_host.blocks import LLAMA_7B, DecoderShape, decoder_graph
from tests.helpers import (TOL_BF16, assert_close, from_pages, page_table, seeded_graph_inputs,
                           to_device_bytes, to_pages)

SMALL = DecoderShape(256, 4, 2, 64, 512, 300, 1)


def _paired(shape, batch, seq, max_len, page, fill, fmt="w4g32", layers=1, spare=3, head="logits",
            pos=None, seed=5):
    """The contiguous graph with its seeded inputs, and the paged graph with
    the same values scattered into shuffled pages (spare unused pages of
    noise per sequence).  max_len is a whole number of pages."""
    assert max_len % page == 0
    gc, hc = decoder_graph(shape, batch=batch, seq=seq, max_len=max_len, fmt=fmt, layers=layers, head=head)
    vals = seeded_graph_inputs(gc, cache_fill=fill)
    vals[hc.tokens] = ora.uniform_i32(2, batch * seq, 0, shape.vocab)
    if pos is None:
        pos = (np.array([fill - i for i in range(batch)], np.int32) if seq == 1
               else np.tile(np.arange(seq, dtype=np.int32), batch))
    vals[hc.pos] = pos
    pps = max_len // page
    npages = batch * (pps + spare)
    gp, hp = decoder_graph(shape, batch=batch, seq=seq, max_len=max_len, fmt=fmt, layers=layers, head=head,
                           kv_page=page, kv_pages=npages)
    table = page_table(batch, pps, npages, seed=seed)
    pvals = {}
    for i, v in enumerate(gp.values):
        if v.producer is None and v.name.endswith("pages"):
            pvals[i] = to_pages(vals[gc.values.index(next(w for w in gc.values if w.name ==
                                                          v.name.replace("pages", "cache")))],
                                table, npages, fill_seed=11 + i)
    for i, v in enumerate(gc.values):
        if v.producer is None and not v.name.endswith("cache") and i in vals:
            j = next(k for k, w in enumerate(gp.values) if w.name == v.name and w.producer is None)
            pvals[j] = vals[i]
    pvals[hp.block_table] = table
    return (gc, hc, vals), (gp, hp, pvals, table)


def _copy(d):
    return {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in d.items()}


def _caches(g, vals_after, suffix):
    return {v.name: vals_after[i] for i, v in enumerate(g.values) if v.name.endswith(suffix) and i in vals_after}


@pytest.mark.parametrize("seq,page", [(1, 16), (1, 32), (24, 16), (24, 64)])
def test_oracle_paged_equals_contiguous(seq, page):
    max_len = 64
    (gc, hc, vals), (gp, hp, pvals, table) = _paired(SMALL, 3, seq, max_len, page, 40 if seq == 1 else 0)
    vc, vp = _copy(vals), _copy(pvals)
    want = graph_eval.evaluate(gc, vc)[hc.out]
    got = graph_eval.evaluate(gp, vp)[hp.out]
    assert np.array_equal(got, want)
    cont = _caches(gc, vc, "cache")
    for name, pool in _caches(gp, vp, "pages").items():
        assert np.array_equal(from_pages(pool, table), cont[name.replace("pages", "cache")]), name


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _run(plugin, g, host):
    arena, bufs = {}, []
    for i, v in enumerate(g.values):
        if v.producer is None and i in host:
            b = plugin.upload(v.dtype, v.dims, to_device_bytes(v, host[i]))
            bufs.append(b)
            arena[i] = Device(b)
    exe = plugin.compile(g)
    assert exe is not None, "the plugin declined the graph"
    try:
        exe.run(arena, every_value=False)
        out = {o: np.array(arena[o]) for o in g.outputs}
        caches = {v.name: bytes(arena[i].buffer.read()) for i, v in enumerate(g.values)
                  if (v.name.endswith("cache") or v.name.endswith("pages")) and i in arena}
    finally:
        exe.free()
        for b in bufs:
            b.release()
    return out, caches


def _bf16(raw, dims):
    return ora.from_bf16(np.frombuffer(raw, np.uint16).reshape(dims))


def _check_pair(plugin, shape, batch, seq, max_len, page, fill, layers=1, pos=None, oracle=False):
    (gc, hc, vals), (gp, hp, pvals, table) = _paired(shape, batch, seq, max_len, page, fill, layers=layers,
                                                    pos=pos)
    oc, cc = _run(plugin, gc, vals)
    op, cp = _run(plugin, gp, pvals)
    assert np.array_equal(np.asarray(op[hp.out]), np.asarray(oc[hc.out])), "paged output differs from contiguous"
    for name, raw in cp.items():
        v = next(w for w in gp.values if w.name == name)
        cname = name.replace("pages", "cache")
        cv = next(w for w in gc.values if w.name == cname)
        got = from_pages(_bf16(raw, v.dims), table)
        assert np.array_equal(got, _bf16(cc[cname], cv.dims)), f"{name}: appended rows differ"
    if oracle:
        ref = graph_eval.evaluate(gp, _copy(pvals))[hp.out]
        assert_close(ora.from_bf16(np.asarray(op[hp.out]).view(np.uint16)), ref, TOL_BF16, "paged logits")


@pytest.mark.gpu
@pytest.mark.parametrize("page", [16, 128, 1024])
def test_paged_decode_is_bit_identical_to_contiguous(cuda, plugin, page):
    """7B-shape decode, batch 4, 2048 cached positions: the fused q/k/v GEMV
    appends through the table and the tensor-core decode attention reads
    through it (splits of 64-position multiples, so slabs stay inside pages)."""
    _check_pair(plugin, LLAMA_7B, 4, 1, 2176 if page < 1024 else 3072, page, 2048, oracle=page == 16)


@pytest.mark.gpu
@pytest.mark.parametrize("page", [16, 64, 256])
def test_paged_prefill_is_bit_identical_to_contiguous(cuda, plugin, page):
    """Prefill of 2 x 320 tokens (three 128-position KV tiles, the last
    partial): the append kernel writes through the table and the tcgen05
    attention loads K/V tiles page by page (boxes of min(page, 128) rows)."""
    shape = DecoderShape(1024, 8, 8, 128, 2816, 512, 1)
    _check_pair(plugin, shape, 2, 320, 512, page, 0, oracle=page == 16)


@pytest.mark.gpu
def test_paged_decode_with_ragged_lengths_and_unmapped_tail_pages(cuda, plugin):
    """Continuous batching: sequences at different lengths, each with only
    the pages its positions reach mapped (the rest of its table row is -1)."""
    shape, batch, page, max_len = LLAMA_7B, 4, 16, 1024
    pos = np.array([1000, 17, 511, 0], np.int32)
    gp, hp = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", layers=1, head="logits",
                           kv_page=page, kv_pages=batch * max_len // page)
    host = seeded_graph_inputs(gp)
    host[hp.tokens] = ora.uniform_i32(2, batch, 0, shape.vocab)
    host[hp.pos] = pos
    table = page_table(batch, max_len // page, batch * max_len // page)
    for b in range(batch):
        table[b, pos[b] // page + 1:] = -1
    host[hp.block_table] = table
    out, _ = _run(plugin, gp, host)
    ref = graph_eval.evaluate(gp, _copy(host))[hp.out]
    assert_close(ora.from_bf16(np.asarray(out[hp.out]).view(np.uint16)), ref, TOL_BF16, "ragged paged logits")


@pytest.mark.gpu
def test_missing_page_is_an_invalid_argument_not_a_fault(cuda, plugin):
    """A table entry that a position needs and that names no page of the pool
    is reported (error word 6) and nothing outside the pool is touched."""
    shape, batch, page, max_len = SMALL, 2, 16, 64
    gp, hp = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", layers=1, head="logits",
                           kv_page=page, kv_pages=8)
    host = seeded_graph_inputs(gp)
    host[hp.tokens] = ora.uniform_i32(2, batch, 0, shape.vocab)
    host[hp.pos] = np.array([40, 20], np.int32)
    table = page_table(batch, max_len // page, 8)
    bad = table.copy()
    bad[0, 1] = 1 << 20
    host[hp.block_table] = bad
    with pytest.raises(StrataError) as e:
        _run(plugin, gp, host)
    assert e.value.code == -3 and "block-table" in str(e.value)
    host[hp.block_table] = table  # the context stays usable
    _run(plugin, gp, host)
