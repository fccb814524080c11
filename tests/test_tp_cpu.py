"""Tensor parallelism without a GPU: two gloo ranks each run their shard graph
on the oracle, all-reducing after o_proj and down_proj, and must reproduce the
unsharded decoder step (the host-side sharding and graph construction that
bench.py --gpus N and the plugin's fused::all_reduce rely on)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tests.conftest import PKG, ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path, fmt="w4g32", page=0):
    """One rank of a tensor-parallel decode step in weight format ``fmt``,
    with page pools of ``page`` positions (contiguous caches when 0).  Every
    rank also runs the unsharded step and checks its caches after the step
    (read back through the block table when paged) against its kv heads of
    the unsharded caches: exactly in layer 0, within the bf16 all-reduce
    tolerance after it.  Rank 0 saves both steps' logits."""
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    from oracle import graph_eval, oracle as ora
    from strata_host.blocks import DecoderShape, decoder_graph, shard_layer
    from tests.helpers import from_pages, page_table, seeded_graph_inputs, to_pages

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shape = DecoderShape(256, 4, 2, 64, 512, 100, 2)
    batch, max_len, fill = 2, 48, 30
    full_g, full_hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt=fmt, head="logits")
    full = seeded_graph_inputs(full_g, cache_fill=fill)
    ids = ora.uniform_i32(2, batch, 0, shape.vocab)
    pos = np.array([fill, fill - 1], np.int32)
    full[full_hd.tokens], full[full_hd.pos] = ids, pos

    paged = {}
    if page:
        pps, npages = max_len // page, batch * (max_len // page) + 3
        paged = {"kv_page": page, "kv_pages": npages}
        table = page_table(batch, pps, npages, seed=9)
    g, hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt=fmt, head="logits",
                          tp_rank=rank, tp_world=world, **paged)
    inputs = {hd.tokens: ids, hd.pos: pos, hd.embed_table: full[full_hd.embed_table],
              hd.final_norm: full[full_hd.final_norm], hd.lm_w: full[full_hd.lm_w], hd.lm_s: full[full_hd.lm_s]}
    if page:
        inputs[hd.block_table] = table
    for li in range(shape.layers):
        layer_full = {k: full[v] for k, v in full_hd.layers[li].ids.items()}
        if page:
            for c in ("k_cache", "v_cache"):
                layer_full[c] = to_pages(layer_full[c], table, npages, fill_seed=21 + li)
        shard = shard_layer(layer_full, shape, fmt, rank, world)
        for k, v in hd.layers[li].ids.items():
            dims = tuple(g.values[v].dims)
            if g.values[v].dtype.element == graph_eval.F4E2M1_E:  # two codes per byte
                dims = dims[:-1] + ((dims[-1] + 1) // 2,)
            assert shard[k].shape == dims, (k, shard[k].shape, dims)
            inputs[v] = shard[k]

    def all_reduce(_name, x):
        t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return ora.round_bf16(t.numpy())

    vals = graph_eval.evaluate(g, inputs, all_reduce=all_reduce)
    ref = graph_eval.evaluate(full_g, {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in full.items()})
    gl = shape.kv_heads // world
    for li in range(shape.layers):
        for c in ("k_cache", "v_cache"):
            mine = vals[hd.layers[li].ids[c]]
            if page:
                mine = from_pages(mine, table)
            want = ref[full_hd.layers[li].ids[c]][:, rank * gl:(rank + 1) * gl]
            if li == 0:  # same normed input, same rows of k/v_proj: exact
                assert np.array_equal(mine, want), f"rank {rank} layer {li} {c} after the step"
            else:  # the input went through the bf16 all-reduce of layer 0
                err = float(np.max(np.abs(mine - want)) / np.max(np.abs(want)))
                assert err <= 2e-2, f"rank {rank} layer {li} {c}: {err:.3e}"
    if rank == 0:
        np.save(result_path, np.stack([vals[hd.out], ref[full_hd.out]]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("fmt,page", [("w4g32", 0), ("w4g32", 16), ("mxfp8", 0), ("mxfp4", 16)])
def test_two_rank_tensor_parallel_step_matches_unsharded(tmp_path, fmt, page):
    """Column-parallel q/k/v/gate/up, row-parallel o/down with a sum over the
    ranks, for int4 and MX weights (codes and E8M0 scale groups sliced along
    K) and for page pools sliced by kv head under one block table."""
    path = str(tmp_path / "tp.npy")
    mp.start_processes(_worker, args=(2, _free_port(), path, fmt, page), nprocs=2, join=True,
                       start_method="spawn")
    got, want = np.load(path)
    err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    assert err <= 2e-2, f"tensor-parallel logits differ from unsharded by {err:.3e}"


@pytest.mark.parametrize("fmt", ["w4g32", "mxfp8", "mxfp4"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ffn_shards_cover_the_ffn_in_whole_units(world, fmt):
    """The 7B FFN (11008) at 8 ranks splits 4 x 1408 + 4 x 1344 for int4
    (even int4 group counts for every down_proj shard) and 6 x 1408 +
    2 x 1280 for MX (K a multiple of 128 for every down_proj shard), and the
    shards of gate/up rows and down_proj codes / scales concatenate back to
    the full matrices."""
    import numpy as np

    from strata_host.blocks import LLAMA_7B, DecoderShape, ffn_shard, ffn_unit, shard_layer, weight_shapes
    shape = DecoderShape(256, 8, 8, 32, 11008, 0, 1)
    unit = ffn_unit(fmt)
    assert unit == (64 if fmt == "w4g32" else 128)
    full = {}
    for name, (dt, dims) in weight_shapes(shape, fmt).items():
        dims = tuple(dims)
        if fmt == "mxfp4" and name[0] == "w":  # E2M1 codes are stored two per byte
            dims = dims[:-1] + (dims[-1] // 2,)
        full[name] = np.arange(int(np.prod(dims)), dtype=np.int64).reshape(dims)
    shards = [shard_layer(full, shape, fmt, r, world) for r in range(world)]
    for r in range(world):
        f0, fn = ffn_shard(shape.ffn, world, r, unit)
        assert fn % unit == 0
        ws = weight_shapes(shape, fmt, world, r)
        for name in ("wg", "sg", "wu", "su", "wd", "sd"):
            want = tuple(ws[name][1])
            if fmt == "mxfp4" and name[0] == "w":
                want = want[:-1] + (want[-1] // 2,)
            assert shards[r][name].shape == want, (name, r)
    for name, axis in (("wg", 0), ("sg", 0), ("wu", 0), ("su", 0), ("wd", 1), ("sd", 1)):
        assert np.array_equal(np.concatenate([s[name] for s in shards], axis=axis), full[name]), name
    want7b = [1408] * 4 + [1344] * 4 if unit == 64 else [1408] * 6 + [1280] * 2
    assert [ffn_shard(LLAMA_7B.ffn, 8, r, unit)[1] for r in range(8)] == want7b


def _worker_argmax(rank, world, port, result_path):
    """A vocabulary-parallel argmax head: each rank holds its rows of the
    lm_head and fused::vocab_argmax gathers the ranks' logits in rank order.
    On the same shards and hidden states, the replicated logits head gives the
    logits whose argmax the distributed ids must equal exactly."""
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    from oracle import graph_eval, oracle as ora
    from strata_host.blocks import DecoderShape, decoder_graph, shard_layer, shard_lm_head, vocab_shard
    from tests.helpers import seeded_graph_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shape = DecoderShape(256, 4, 2, 64, 512, 200, 2)
    batch, max_len, fill = 3, 40, 30
    full_g, full_hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", head="logits")
    full = seeded_graph_inputs(full_g, cache_fill=fill)
    ids = ora.uniform_i32(2, batch, 0, shape.vocab)
    pos = np.array([fill, fill - 1, fill - 2], np.int32)

    def all_reduce(_name, x):
        t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return ora.round_bf16(t.numpy())

    def all_gather(_name, x):
        # Shards differ in width (the last one is short), so each is padded to
        # the widest before the gather and trimmed after it.
        widths = [vocab_shard(shape.vocab, world, r)[1] for r in range(world)]
        x = np.ascontiguousarray(x, np.float32)
        pad = np.zeros((x.shape[0], max(widths)), np.float32)
        pad[:, :x.shape[1]] = x
        parts = [torch.empty(pad.shape) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pad))
        return [q.numpy()[:, :w] for q, w in zip(parts, widths)]

    outs = {}
    for head in ("argmax", "logits"):
        g, hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", head=head,
                              tp_rank=rank, tp_world=world)
        lm_w, lm_s = full[full_hd.lm_w], full[full_hd.lm_s]
        if head == "argmax":
            lm_w, lm_s = shard_lm_head(lm_w, lm_s, shape.vocab, world, rank)
            assert lm_w.shape == tuple(g.values[hd.lm_w].dims)
        inputs = {hd.tokens: ids, hd.pos: pos, hd.embed_table: full[full_hd.embed_table],
                  hd.final_norm: full[full_hd.final_norm], hd.lm_w: lm_w, hd.lm_s: lm_s}
        for li in range(shape.layers):
            layer_full = {k: full[v] for k, v in full_hd.layers[li].ids.items()}
            shard = shard_layer(layer_full, shape, "w4g32", rank, world)
            for k, v in hd.layers[li].ids.items():
                inputs[v] = shard[k]
        outs[head] = graph_eval.evaluate(g, inputs, all_reduce=all_reduce, all_gather=all_gather)[hd.out]
    got = np.asarray(outs["argmax"], np.int32)
    want = ora.argmax(outs["logits"])
    every = [torch.zeros(batch, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(every, torch.from_numpy(got))
    if rank == 0:
        np.save(result_path, np.stack([got, want] + [e.numpy() for e in every]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_vocab_parallel_argmax_matches_the_replicated_head(tmp_path):
    path = str(tmp_path / "vargmax.npy")
    mp.start_processes(_worker_argmax, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    rows = np.load(path)
    got, want = rows[0], rows[1]
    assert np.array_equal(got, want), (got, want)
    for other in rows[2:]:
        assert np.array_equal(other, got), "ranks disagree on the next-token ids"


@pytest.mark.parametrize("vocab,world", [(32000, 2), (32000, 8), (32000, 3), (200, 2), (50, 8)])
def test_vocab_shards_tile_the_vocabulary(vocab, world):
    """Shards are contiguous, in rank order, cover every id once, and every
    shard but the one that ends the vocabulary is a multiple of 16 rows."""
    from strata_host.blocks import vocab_shard
    nxt = 0
    for r in range(world):
        v0, n = vocab_shard(vocab, world, r)
        assert v0 == nxt and n >= 0
        if v0 + n < vocab:
            assert n % 16 == 0
        nxt = v0 + n
    assert nxt == vocab


def test_vocab_argmax_head_refuses_an_empty_shard():
    """A vocabulary of 50 over 8 ranks leaves ranks 4-7 without lm_head rows."""
    from strata_host.blocks import DecoderShape, decoder_graph
    with pytest.raises(ValueError):
        decoder_graph(DecoderShape(64, 2, 2, 32, 128, 50, 1), batch=1, seq=1, max_len=16, fmt="w4g32",
                      head="argmax", tp_rank=7, tp_world=8)
