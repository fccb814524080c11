"""Evaluate a Strata subgraph on the CPU oracle, node by node.

TEST INFRASTRUCTURE ONLY (the checker for graph-level parity tests).

Semantics follow the reference CPU executor (crates/ferrite-strata-cpu/src/
backend.rs:187-304): steps run in node order and only the declared outputs
are published.  Every bf16 value is rounded to bf16 when it is produced (each
graph value has one dtype), with f32 arithmetic inside each op.  The GPU may
fuse ops and skip an intermediate rounding; the parity tolerance covers that.

Arena values are numpy arrays: f32 for F32 and BF16 values (BF16 held as
bf16-representable f32, or passed in raw as uint16), int32 for I32, uint8 /
int8 for quantised codes.
"""
from __future__ import annotations

import numpy as np

from . import oracle as ora

F32_E, BF16_E, I32_E, F4E2M1_E = 4, 14, 8, 13


def _is_bf16(dt) -> bool:
    return dt.element == BF16_E and dt.quant_kind == 0


def _norm_in(v, arr):
    if _is_bf16(v.dtype):
        a = np.asarray(arr)
        return ora.from_bf16(a) if a.dtype == np.uint16 else ora.round_bf16(a)
    if v.dtype.element == F32_E:
        return np.asarray(arr, dtype=np.float32)
    if v.dtype.element == I32_E:
        return np.asarray(arr, dtype=np.int32)
    return np.asarray(arr)


def _threads() -> int:
    # The threaded oracle kernels give every output element to one thread,
    # which accumulates it in the same k order as the single-threaded ones,
    # so the results are identical; threads only shorten large parity cases.
    return ora.max_threads()


def evaluate(graph, inputs: dict, all_reduce=None, all_gather=None) -> dict:
    """Run `graph` on the oracle.  `inputs` maps value id -> array; KV caches
    are updated in place in the returned dict.  `all_reduce(name, x)` sums
    over tensor-parallel ranks (identity when None); `all_gather(name, x)`
    returns every rank's x in rank order (a one-element list when None)."""
    vals: dict[int, np.ndarray] = {}
    for i, v in enumerate(graph.values):
        if v.producer is None and i in inputs:
            dims = tuple(v.dims)
            if v.dtype.element == F4E2M1_E:  # codes packed two per byte along the last axis
                dims = dims[:-1] + ((dims[-1] + 1) // 2,)
            vals[i] = _norm_in(v, inputs[i]).reshape(dims)

    def out_dt(n, i=0):
        return graph.values[n.outputs[i]].dtype

    for n in graph.nodes:
        op = n.op
        ins = [vals[i] for i in n.inputs]
        dt = out_dt(n) if n.outputs else None
        shape = graph.values[n.outputs[0]].dims if n.outputs else ()
        k = op.kind
        pid = op.pattern_id
        res = None
        if k in ("add", "mul"):
            res = ora.elementwise(k, ins[0], ins[1], shape)
        elif k == "matmul":
            res = ora.matmul(ins[0], ins[1])
        elif k in ("log", "exp", "gelu"):
            res = {"log": ora.log, "exp": ora.exp, "gelu": ora.gelu}[k](ins[0])
        elif k == "softmax":
            res = ora.softmax(ins[0])
        elif k == "layer_norm":
            res = ora.layer_norm(ins[0], vals[op.gamma], vals[op.beta], op.eps)
        elif k == "linear":
            x = ins[0].reshape(-1, ins[0].shape[-1])
            res = ora.linear(x, vals[op.weight], vals[op.bias] if op.bias is not None else None)
        elif k == "reshape":
            res = ins[0].reshape(shape)
        elif k == "transpose":
            res = ora.transpose2(ins[0])
        elif k == "expand":
            res = ora.broadcast_to(ins[0], shape)
        elif k == "slice":
            res = ora.slice_cols(ins[0], op.start, op.end, op.stride)
        elif k == "input":
            continue
        elif pid == "fused::linear_w4g32":
            x = ins[0].reshape(-1, ins[0].shape[-1])
            res = ora.linear_w4g32(x, ins[1], ora.to_bf16(ins[2]), threads=_threads())
        elif pid in ("fused::linear_mxfp8", "fused::linear_mxfp4"):
            x = ins[0].reshape(-1, ins[0].shape[-1])
            res = ora.linear_mx(x, ins[1], ins[2], pid.rsplit("_", 1)[1], threads=_threads())
        elif pid == "fused::linear_w8pc":
            x = ins[0].reshape(-1, ins[0].shape[-1])
            res = ora.linear_w8pc(x, ins[1], ins[2], threads=_threads())
        elif pid == "fused::rms_norm":
            res = ora.rms_norm(ins[0], ins[1], float(n.attrs.get("eps", 1e-5)))
        elif pid == "fused::rope":
            res = ora.rope(ins[0], ins[1], int(n.attrs["head_dim"]), float(n.attrs.get("theta", 10000.0)))
        elif pid == "fused::swiglu":
            res = ora.swiglu(ins[0], ins[1])
        elif pid == "fused::attention" and int(n.attrs.get("page_size", 0)) > 0:
            # Paged caches: page pools [pages, G, page_size, d] and a block
            # table [B, pages_per_seq]; position p of sequence s is row
            # p % page_size of page table[s, p // page_size].  The append
            # writes each new row into its page, then attention reads each
            # sequence's pages in table order, exactly as the contiguous
            # cache below.
            q, kn, vn, kp, vp, pos, table = ins[:7]
            H, G, d = int(n.attrs["num_heads"]), int(n.attrs["num_kv_heads"]), int(n.attrs["head_dim"])
            ps = int(n.attrs["page_size"])
            B, pps = table.shape
            rows = q.size // (H * d)
            seq = np.arange(rows, dtype=np.int32) // (rows // B)
            knr = kn.reshape(rows, G, d)
            vnr = vn.reshape(rows, G, d)
            for r in range(rows):
                p = int(pos[r])
                if 0 <= p < pps * ps:
                    pg = int(table[seq[r], p // ps])
                    if 0 <= pg < kp.shape[0]:
                        kp[pg, :, p % ps, :] = knr[r]
                        vp[pg, :, p % ps, :] = vnr[r]
            kc = np.zeros((B, G, pps * ps, d), kp.dtype)
            vc = np.zeros_like(kc)
            for s in range(B):
                for lp in range(pps):
                    pg = int(table[s, lp])
                    if 0 <= pg < kp.shape[0]:
                        kc[s, :, lp * ps:(lp + 1) * ps, :] = kp[pg]
                        vc[s, :, lp * ps:(lp + 1) * ps, :] = vp[pg]
            res = ora.attention(q, kc, vc, seq, pos, H, G, d, threads=_threads())
        elif pid == "fused::attention":
            q, kn, vn, kc, vc, pos = ins[:6]
            H, G, d = int(n.attrs["num_heads"]), int(n.attrs["num_kv_heads"]), int(n.attrs["head_dim"])
            B = kc.shape[0]
            rows = q.size // (H * d)
            per = rows // B
            seq = np.arange(rows, dtype=np.int32) // per
            knr = kn.reshape(rows, G, d)
            vnr = vn.reshape(rows, G, d)
            for r in range(rows):
                p = int(pos[r])
                if 0 <= p < kc.shape[2]:
                    kc[seq[r], :, p, :] = knr[r]
                    vc[seq[r], :, p, :] = vnr[r]
            res = ora.attention(q, kc, vc, seq, pos, H, G, d, threads=_threads())
        elif pid == "fused::embed":
            res, _rc = ora.embed(ins[0], ins[1])
        elif pid == "fused::argmax":
            res = ora.argmax(ins[0])
        elif pid == "fused::vocab_argmax":
            # The argmax over the vocabulary split by rows between the ranks:
            # the same rules as fused::argmax over the rank-ordered
            # concatenation of the shards (NaN skipped, lowest id on ties, 0
            # for a row with no number); alone, this shard's ids start at
            # vocab_offset.
            shard = np.asarray(ins[0], np.float32).reshape(-1, ins[0].shape[-1])
            if all_gather is None:
                ids = ora.argmax(shard).astype(np.int64)
                has = ~np.all(np.isnan(shard), axis=1)
                res = np.where(has, ids + int(n.attrs.get("vocab_offset", 0)), 0).astype(np.int32)
            else:
                res = ora.argmax(np.concatenate(all_gather(n.name, shard), axis=1))
        elif pid == "fused::last_token":
            B = graph.values[n.outputs[0]].dims[0]
            x = ins[0].reshape(B, -1, ins[0].shape[-1])
            res = x[:, -1, :]
        elif pid == "fused::all_reduce":
            res = ins[0] if all_reduce is None else all_reduce(n.name, ins[0])
        elif pid == "fused::quantize_w4g32":
            c, s = ora.quant_w4g32(ins[0])
            vals[n.outputs[0]] = c
            vals[n.outputs[1]] = ora.from_bf16(s)
            continue
        elif pid == "fused::quantize_w8pc":
            c, s = ora.quant_w8pc(ins[0])
            vals[n.outputs[0]] = c
            vals[n.outputs[1]] = s
            continue
        elif pid == "fused::dequantize_w4g32":
            res = ora.dequant_w4g32(ins[0], ora.to_bf16(ins[1]))
        elif pid == "fused::dequantize_w8pc":
            res = ora.dequant_w8pc(ins[0], ins[1])
        else:
            raise NotImplementedError(f"no oracle for `{pid or k}`")
        res = np.asarray(res)
        if dt is not None and _is_bf16(dt):
            res = ora.round_bf16(res)
        vals[n.outputs[0]] = res.reshape(shape)
    return vals
