"""One rank of the multi-GPU tensor-parallel parity check, started under
torchrun by tests/test_gpu_tp.py.

Every rank builds the same full (unsharded) weights of a small GQA decoder
from fixed seeds, keeps its own shard (column-parallel q/k/v/gate/up,
row-parallel o/down), joins the plugin's NCCL group and runs one step through
the plugin: a decode step of 4 rows (the residual all-reduces run fused with
the add and RMSNorm that follow them, over NVLink) or, with ``prefill`` as the
second argument, a prefill of 2 x 40 rows (more rows than the fused kernel
takes: NCCL, then the add and the norm).  The step runs three times and every
run must give the same logits (the exchange's flags and slots alternate
between runs).  Rank 0 writes its logits and the oracle's logits of the
unsharded step to the path given on the command line.

With ``argmax`` as the second argument the step is the decode step with the
vocabulary-parallel argmax head: each rank holds its rows of the lm_head, the
graph also returns the rank's logits shard, and the ranks' ids must be equal
to each other and to the argmax of the shards gathered in rank order (exact).
Rank 0 then writes its ids, that argmax and every rank's ids."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ferrite-strata_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch.distributed as dist  # noqa: E402

from oracle import graph_eval, oracle as ora  # noqa: E402
from strata_host import BF16, Device, Plugin  # noqa: E402
from strata_host.blocks import DecoderShape, decoder_graph, shard_layer, shard_lm_head, vocab_shard  # noqa: E402
from tests.helpers import seeded_graph_inputs, to_device_bytes  # noqa: E402

# 16 query / 8 kv heads of 128, FFN 11008 (the 7B FFN: at 8 ranks its shards are 1408 and 1344
# features, so the uneven FFN split is exercised).
SHAPE = DecoderShape(2048, 16, 8, 128, 11008, 512, 2)
MAX_LEN = 136


def main(out_path, mode):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    os.environ["STRATA_B200_DEVICE"] = str(local)

    batch, seq, fill = (2, 40, 0) if mode == "prefill" else (4, 1, 128)
    full_g, full_hd = decoder_graph(SHAPE, batch=batch, seq=seq, max_len=MAX_LEN, fmt="w4g32", head="logits")
    full = seeded_graph_inputs(full_g, cache_fill=fill)
    full[full_hd.tokens] = ora.uniform_i32(2, batch * seq, 0, SHAPE.vocab)
    if seq == 1:
        full[full_hd.pos] = np.array([fill - i for i in range(batch)], np.int32)
    else:
        full[full_hd.pos] = np.tile(np.arange(seq, dtype=np.int32), batch)

    head = "argmax" if mode == "argmax" else "logits"
    g, hd = decoder_graph(SHAPE, batch=batch, seq=seq, max_len=MAX_LEN, fmt="w4g32", head=head,
                          tp_rank=rank, tp_world=world)
    lm_w, lm_s = full[full_hd.lm_w], full[full_hd.lm_s]
    logits_id = None
    if head == "argmax":
        lm_w, lm_s = shard_lm_head(lm_w, lm_s, SHAPE.vocab, world, rank)
        logits_id = g.nodes[-1].inputs[0]
        g.outputs.append(logits_id)
    host = {hd.tokens: full[full_hd.tokens], hd.pos: full[full_hd.pos],
            hd.embed_table: full[full_hd.embed_table], hd.final_norm: full[full_hd.final_norm],
            hd.lm_w: lm_w, hd.lm_s: lm_s}
    for li in range(SHAPE.layers):
        shard = shard_layer({k: full[v] for k, v in full_hd.layers[li].ids.items()}, SHAPE, "w4g32", rank, world)
        for k, v in hd.layers[li].ids.items():
            host[v] = shard[k]

    plugin = Plugin(os.path.join(PKG, "libstrata_b200.so"))
    uid = [plugin.tp_unique_id() if rank == 0 else b""]
    dist.broadcast_object_list(uid, 0)
    plugin.tp_init(rank, world, uid[0])

    arena, bufs = {}, []
    for i, v in enumerate(g.values):
        if v.producer is None and i in host:
            b = plugin.upload(v.dtype, v.dims, to_device_bytes(v, host[i]))
            bufs.append(b)
            arena[i] = Device(b)
    exe = plugin.compile(g)
    assert exe is not None, "the plugin declined the shard graph"
    runs = []
    for _ in range(3):
        exe.run(arena)
        runs.append(np.array(arena[hd.out]))
    shard = None
    if logits_id is not None:
        shard = ora.from_bf16(np.array(arena[logits_id]).view(np.uint16))
    for i, r in enumerate(runs[1:], 1):
        assert np.array_equal(r, runs[0]), f"rank {rank}: run {i} differs from run 0"
    got = runs[0]
    if g.values[hd.out].dtype == BF16:
        got = ora.from_bf16(got.view(np.uint16))
    exe.free()
    for b in bufs:
        b.release()
    plugin.close()

    if head == "argmax":
        import torch
        width = vocab_shard(SHAPE.vocab, world, 0)[1]
        pad = np.zeros((batch, width), np.float32)
        pad[:, :shard.shape[1]] = shard
        parts = [torch.empty(batch, width) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pad))
        ids = [torch.empty(batch, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(ids, torch.from_numpy(np.asarray(got, np.int32)))
        if rank == 0:
            logits = np.concatenate([p.numpy()[:, :vocab_shard(SHAPE.vocab, world, r)[1]]
                                     for r, p in enumerate(parts)], axis=1)
            np.save(out_path, np.stack([np.asarray(got, np.int32), ora.argmax(logits)] +
                                       [i.numpy() for i in ids]))
    elif rank == 0:
        want = graph_eval.evaluate(full_g, full)[full_hd.out]
        np.save(out_path, np.stack([np.asarray(got, np.float32), np.asarray(want, np.float32)]))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "decode")
