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


def _worker(rank, world, port, result_path):
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    from oracle import graph_eval, oracle as ora
    from strata_host.blocks import DecoderShape, decoder_graph, shard_layer
    from tests.helpers import seeded_graph_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shape = DecoderShape(256, 4, 2, 64, 512, 100, 2)
    batch, max_len, fill = 2, 40, 30
    full_g, full_hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", head="logits")
    full = seeded_graph_inputs(full_g, cache_fill=fill)
    ids = ora.uniform_i32(2, batch, 0, shape.vocab)
    pos = np.array([fill, fill - 1], np.int32)
    full[full_hd.tokens], full[full_hd.pos] = ids, pos

    g, hd = decoder_graph(shape, batch=batch, seq=1, max_len=max_len, fmt="w4g32", head="logits",
                          tp_rank=rank, tp_world=world)
    inputs = {hd.tokens: ids, hd.pos: pos, hd.embed_table: full[full_hd.embed_table],
              hd.final_norm: full[full_hd.final_norm], hd.lm_w: full[full_hd.lm_w], hd.lm_s: full[full_hd.lm_s]}
    for li in range(shape.layers):
        layer_full = {k: full[v] for k, v in full_hd.layers[li].ids.items()}
        shard = shard_layer(layer_full, shape, "w4g32", rank, world)
        for k, v in hd.layers[li].ids.items():
            assert shard[k].shape == tuple(g.values[v].dims), (k, shard[k].shape, g.values[v].dims)
            inputs[v] = shard[k]

    def all_reduce(_name, x):
        t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return ora.round_bf16(t.numpy())

    got = graph_eval.evaluate(g, inputs, all_reduce=all_reduce)[hd.out]
    if rank == 0:
        want = graph_eval.evaluate(full_g, full)[full_hd.out]
        np.save(result_path, np.stack([got, want]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_tensor_parallel_step_matches_unsharded(tmp_path):
    path = str(tmp_path / "tp.npy")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    got, want = np.load(path)
    err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    assert err <= 2e-2, f"tensor-parallel logits differ from unsharded by {err:.3e}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ffn_shards_cover_the_ffn_with_even_group_counts(world):
    """The 7B FFN (11008) at 8 ranks splits 4 x 1408 + 4 x 1344 (even int4 group counts for every
    down_proj shard), and the shards of gate/up rows and down_proj codes / scales concatenate
    back to the full matrices."""
    import numpy as np

    from strata_host.blocks import LLAMA_7B, DecoderShape, ffn_shard, shard_layer, weight_shapes
    shape = DecoderShape(256, 8, 8, 32, 11008, 0, 1)
    full = {}
    for name, (dt, dims) in weight_shapes(shape, "w4g32").items():
        full[name] = np.arange(int(np.prod(dims)), dtype=np.int64).reshape(dims)
    shards = [shard_layer(full, shape, "w4g32", r, world) for r in range(world)]
    for r in range(world):
        f0, fn = ffn_shard(shape.ffn, world, r)
        assert fn % 64 == 0 and (fn // 32) % 2 == 0
        ws = weight_shapes(shape, "w4g32", world, r)
        for name in ("wg", "sg", "wu", "su", "wd", "sd"):
            assert shards[r][name].shape == ws[name][1], (name, r)
    for name, axis in (("wg", 0), ("sg", 0), ("wu", 0), ("su", 0), ("wd", 1), ("sd", 1)):
        assert np.array_equal(np.concatenate([s[name] for s in shards], axis=axis), full[name]), name
    assert [ffn_shard(LLAMA_7B.ffn, 8, r)[1] for r in range(8)] == [1408] * 4 + [1344] * 4


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
