"""Decoder-block subgraphs in the Strata IR, ready for the B200 plugin.

The reference IR has no decoder ops (crates/ferrite-strata/src/graph.rs:56-128),
so each one is an ``Op::Custom`` with a vendor pattern id and its parameters in
node attributes (attrs.rs:39-51), and every weight is a node input so that a
subgraph cut keeps it (graph.rs:422-436 remaps only node inputs):

==========================  =========================================  ====================
pattern                     inputs                                     attributes
==========================  =========================================  ====================
fused::linear_w4g32         x bf16 [M,K], codes U8{32} [N,K/2],        bits=4, group_size=32
                            scales bf16 [N,K/32]
fused::linear_w8pc          x bf16 [M,K], codes I8{K} [N,K], f32 [N]   bits=8
fused::linear_mxfp8         x bf16 [M,K], codes f8e4m3 [N,K],          block_size=32
                            scales f8e8m0:mx32 [N,K/32]
fused::linear_mxfp4         x bf16 [M,K], codes f4e2m1:mx32 [N,K]      block_size=32
                            (two per byte), scales f8e8m0:mx32
fused::rms_norm             x [R,C], gamma [C]                         eps
fused::rope                 x [R,H*d], pos I32 [R]                     head_dim, theta
fused::swiglu               gate, up (same shape)
fused::attention            q [R,H*d], k [R,G*d], v [R,G*d],           num_heads,
                            k_cache, v_cache [B,G,L,d], pos I32 [R]    num_kv_heads, head_dim
                            paged: pools [P,G,ps,d], pos, then a       page_size (ps)
                            block table I32 [B, L/ps]
fused::embed                ids I32 [R], table [V,D]
fused::argmax               x [R,C] -> I32 [R] (lowest index on ties)
fused::vocab_argmax         logits shard [R,Vr] -> I32 [R]: the argmax   vocab_offset (id of column 0)
                            over every tensor-parallel rank's shard
fused::all_reduce           x -> sum of x over the tensor-parallel group
fused::last_token           x [B*S,C] -> [B,C], each sequence's last row  tokens_per_seq
==========================  =========================================  ====================

``fused::attention`` appends row r's k/v at ``pos[r]`` of sequence
``r // (R / B)`` in the caches (an in-place update of two inputs) and then
attends over positions ``0..pos[r]``; causality comes from the positions.
Tensor-parallel builds shard q/k/v/gate/up by output column and o/down by
input row, with an all-reduce after o_proj and after down_proj only.  With
the argmax head the lm_head is vocabulary-parallel: each rank holds the rows
``vocab_shard`` gives it and ``fused::vocab_argmax`` combines the ranks'
row maxima into the global next-token ids (the logits head stays replicated).
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .ir import BF16, E2M1, E4M3, E8M0, F32, I32, W4G32, DType, GraphBuilder, Op, w8pc

# MX weight formats: element dtype of the codes (the scales are E8M0, one per
# 32 codes along K).
MX_CODES = {"mxfp8": E4M3, "mxfp4": E2M1}


@dataclass(frozen=True)
class DecoderShape:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    layers: int
    eps: float = 1e-5
    theta: float = 10000.0


# The shapes the benchmark configurations name.
BLOCK_512 = DecoderShape(512, 8, 8, 64, 1408, 0, 1)
LLAMA_7B = DecoderShape(4096, 32, 32, 128, 11008, 32000, 32)
LLAMA_70B = DecoderShape(8192, 64, 8, 128, 28672, 0, 80)


@dataclass
class LayerHandles:
    ids: dict = field(default_factory=dict)   # weight / cache name -> value id


@dataclass
class DecoderHandles:
    tokens: int = -1            # ids I32 [R] (embed=True) or activations [R, D]
    pos: int = -1               # I32 [R]
    layers: list = field(default_factory=list)
    final_norm: int = -1
    lm_w: int = -1
    lm_s: int = -1
    embed_table: int = -1
    out: int = -1               # argmax ids, logits, or the last hidden state
    hidden_out: int = -1
    block_table: int = -1       # paged caches: I32 [batch, pages_per_seq], shared by every layer


def ffn_unit(fmt: str) -> int:
    """Features per FFN slice unit for weight format ``fmt``: 128 for the MX
    formats (their GEMV stages four 32-code scale bytes of a row at a time,
    so a down_proj shard's K is a multiple of 128), else 64 (two int4 groups,
    the int4 GEMV's even group count)."""
    return 128 if fmt in MX_CODES else 64


def ffn_shard(ffn: int, tp_world: int, tp_rank: int, unit: int = 64) -> tuple[int, int]:
    """(first feature, features) of rank tp_rank's slice of the FFN.

    Slices are whole units of ``unit`` features (``ffn_unit`` of the weight
    format) where the FFN allows it, so every rank's down_proj meets the
    tensor-core GEMV's K rule; the first (units % world) ranks take one unit
    more.  The 7B FFN of 11008 at 8 ranks splits as 4 x 1408 + 4 x 1344 in
    64-feature units (instead of 8 x 1376, 43 int4 groups) and as
    6 x 1408 + 2 x 1280 in 128-feature units.  Otherwise the FFN is split
    evenly."""
    t, r = tp_world, tp_rank
    if ffn % unit == 0 and ffn // unit >= t:
        base, extra = divmod(ffn // unit, t)
        return (r * base + min(r, extra)) * unit, (base + (1 if r < extra else 0)) * unit
    if ffn % t:
        raise ValueError("the ffn must divide by the tensor-parallel size")
    return r * (ffn // t), ffn // t


def vocab_shard(vocab: int, tp_world: int, tp_rank: int) -> tuple[int, int]:
    """First vocabulary id and row count of rank ``tp_rank``'s lm_head shard:
    equal shards of a multiple of 16 rows (the GEMV's output tile), the last
    rank taking what remains."""
    per = -(-vocab // (tp_world * 16)) * 16
    v0 = min(tp_rank * per, vocab)
    return v0, min(per, vocab - v0)


def shard_lm_head(w, s, vocab: int, tp_world: int, tp_rank: int):
    """Rank ``tp_rank``'s rows of the full lm_head codes ``w`` and scales ``s``
    (both row-major with one row per vocabulary id, in any weight format)."""
    v0, n = vocab_shard(vocab, tp_world, tp_rank)
    return w[v0:v0 + n].copy(), (None if s is None else s[v0:v0 + n].copy())


def weight_shapes(shape: DecoderShape, fmt: str, tp_world: int = 1, tp_rank: int = 0) -> dict:
    """Per-layer weight tensors (name -> (dtype, dims)) for one rank."""
    D, H, G, d = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim
    t = tp_world
    if H % t or G % t:
        raise ValueError("heads and kv heads must divide by the tensor-parallel size")
    Fr = ffn_shard(shape.ffn, t, tp_rank, ffn_unit(fmt))[1]
    act = F32 if fmt == "f32" else BF16
    mats = {"q": (H // t * d, D), "k": (G // t * d, D), "v": (G // t * d, D), "o": (D, H // t * d),
            "g": (Fr, D), "u": (Fr, D), "d": (D, Fr)}
    out = {"attn_norm": (act, (D,)), "ffn_norm": (act, (D,))}
    for key, (n, k) in mats.items():
        if fmt == "w4g32":
            out["w" + key] = (W4G32, (n, k // 2))
            out["s" + key] = (BF16, (n, k // 32))
        elif fmt == "w8pc":
            out["w" + key] = (w8pc(k), (n, k))
            out["s" + key] = (F32, (n,))
        elif fmt in MX_CODES:
            out["w" + key] = (MX_CODES[fmt], (n, k))
            out["s" + key] = (E8M0, (n, k // 32))
        elif fmt in ("f32", "bf16"):
            out["w" + key] = (act, (n, k))
        else:
            raise ValueError(f"unknown weight format {fmt}")
    return out


def _linear(b: GraphBuilder, x: int, W: dict, key: str, m: int, n: int, fmt: str, act: DType,
            name: str) -> int:
    if fmt == "w4g32":
        return b.node(Op.custom("fused::linear_w4g32"), [x, W["w" + key], W["s" + key]],
                      [(BF16, (m, n))], {"bits": 4, "group_size": 32}, name)[0]
    if fmt == "w8pc":
        return b.node(Op.custom("fused::linear_w8pc"), [x, W["w" + key], W["s" + key]],
                      [(BF16, (m, n))], {"bits": 8}, name)[0]
    if fmt in MX_CODES:
        return b.node(Op.custom(f"fused::linear_{fmt}"), [x, W["w" + key], W["s" + key]],
                      [(BF16, (m, n))], {"block_size": 32}, name)[0]
    return b.node(Op("linear", weight=W["w" + key]), [x], [(act, (m, n))], {}, name)[0]


def decoder_graph(shape: DecoderShape, *, batch: int, seq: int, max_len: int, fmt: str = "w4g32",
                  layers: int | None = None, embed: bool = True, head: str = "argmax",
                  lm_fmt: str | None = None, tp_rank: int = 0, tp_world: int = 1,
                  last_token: bool = False, kv_page: int = 0, kv_pages: int | None = None,
                  name: str = "decoder"):
    """One forward step of ``layers`` decoder blocks over ``batch * seq`` rows.

    ``seq == 1`` is a decode step; ``seq > 1`` a prefill from position 0 (the
    caller fills ``pos``).  ``head``: "argmax" (next-token ids), "logits", or
    "none" (the last hidden state is the output).  ``last_token`` runs the
    head on each sequence's last row only (prefill logits for the next token).
    ``kv_page`` > 0 pages the KV cache: each layer's k/v caches become page
    pools ``[kv_pages, kv_heads, kv_page, head_dim]`` (``kv_pages`` defaults
    to ``batch * ceil(max_len / kv_page)``) and one block table
    ``I32 [batch, ceil(max_len / kv_page)]`` (``block_table``) maps every
    sequence's positions to pages; a sequence's capacity is then a whole
    number of pages.
    """
    layers = shape.layers if layers is None else layers
    act = F32 if fmt == "f32" else BF16
    D, H, G, d = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim
    t = tp_world
    R = batch * seq
    b = GraphBuilder(name)
    hd = DecoderHandles()
    if embed:
        hd.tokens = b.input(I32, (R,), "ids")
        hd.embed_table = b.input(act, (shape.vocab, D), "embed_table")
    else:
        hd.tokens = b.input(act, (R, D), "x")
    hd.pos = b.input(I32, (R,), "pos")
    attn_attrs = {}
    if kv_page:
        pps = -(-max_len // kv_page)
        npages = batch * pps if kv_pages is None else kv_pages
        hd.block_table = b.input(I32, (batch, pps), "block_table")
        attn_attrs = {"page_size": kv_page}
    wshapes = weight_shapes(shape, fmt, t, tp_rank)
    for li in range(layers):
        W = {k: b.input(dt, dims, f"l{li}.{k}") for k, (dt, dims) in wshapes.items()}
        if kv_page:
            W["k_cache"] = b.input(act, (npages, G // t, kv_page, d), f"l{li}.k_pages")
            W["v_cache"] = b.input(act, (npages, G // t, kv_page, d), f"l{li}.v_pages")
        else:
            W["k_cache"] = b.input(act, (batch, G // t, max_len, d), f"l{li}.k_cache")
            W["v_cache"] = b.input(act, (batch, G // t, max_len, d), f"l{li}.v_cache")
        hd.layers.append(LayerHandles(W))
    # Vocabulary-parallel lm_head (argmax head at tensor-parallel size > 1).
    vpar = head == "argmax" and t > 1
    v0, Vr = vocab_shard(shape.vocab, t, tp_rank) if vpar else (0, shape.vocab)
    if vpar and Vr == 0:
        raise ValueError(f"a vocabulary of {shape.vocab} leaves rank {tp_rank} of {t} no lm_head rows")
    if head != "none":
        hd.final_norm = b.input(act, (D,), "final_norm")
        lmf = lm_fmt or fmt
        if lmf == "w4g32":
            hd.lm_w = b.input(W4G32, (Vr, D // 2), "lm_head.w")
            hd.lm_s = b.input(BF16, (Vr, D // 32), "lm_head.s")
        elif lmf == "w8pc":
            hd.lm_w = b.input(w8pc(D), (Vr, D), "lm_head.w")
            hd.lm_s = b.input(F32, (Vr,), "lm_head.s")
        elif lmf in MX_CODES:
            hd.lm_w = b.input(MX_CODES[lmf], (Vr, D), "lm_head.w")
            hd.lm_s = b.input(E8M0, (Vr, D // 32), "lm_head.s")
        else:
            hd.lm_w = b.input(act, (Vr, D), "lm_head.w")

    if embed:
        h = b.node(Op.custom("fused::embed"), [hd.tokens, hd.embed_table], [(act, (R, D))], {}, "embed")[0]
    else:
        h = hd.tokens
    Hl, Gl, Fl = H // t, G // t, ffn_shard(shape.ffn, t, tp_rank, ffn_unit(fmt))[1]
    for li, L in enumerate(hd.layers):
        W = L.ids
        p = f"l{li}."
        n1 = b.node(Op.custom("fused::rms_norm"), [h, W["attn_norm"]], [(act, (R, D))],
                    {"eps": float(shape.eps)}, p + "attn_rms")[0]
        q = _linear(b, n1, W, "q", R, Hl * d, fmt, act, p + "q_proj")
        k = _linear(b, n1, W, "k", R, Gl * d, fmt, act, p + "k_proj")
        v = _linear(b, n1, W, "v", R, Gl * d, fmt, act, p + "v_proj")
        rope_attrs = {"head_dim": d, "theta": float(shape.theta)}
        qr = b.node(Op.custom("fused::rope"), [q, hd.pos], [(act, (R, Hl * d))], rope_attrs, p + "q_rope")[0]
        kr = b.node(Op.custom("fused::rope"), [k, hd.pos], [(act, (R, Gl * d))], rope_attrs, p + "k_rope")[0]
        ains = [qr, kr, v, W["k_cache"], W["v_cache"], hd.pos] + ([hd.block_table] if kv_page else [])
        o = b.node(Op.custom("fused::attention"), ains, [(act, (R, Hl * d))],
                   {"num_heads": Hl, "num_kv_heads": Gl, "head_dim": d, **attn_attrs}, p + "attention")[0]
        a = _linear(b, o, W, "o", R, D, fmt, act, p + "o_proj")
        if t > 1:
            a = b.node(Op.custom("fused::all_reduce"), [a], [(act, (R, D))], {}, p + "o_allreduce")[0]
        h2 = b.node(Op("add"), [h, a], [(act, (R, D))], {}, p + "attn_residual")[0]
        n2 = b.node(Op.custom("fused::rms_norm"), [h2, W["ffn_norm"]], [(act, (R, D))],
                    {"eps": float(shape.eps)}, p + "ffn_rms")[0]
        gt = _linear(b, n2, W, "g", R, Fl, fmt, act, p + "gate_proj")
        up = _linear(b, n2, W, "u", R, Fl, fmt, act, p + "up_proj")
        s = b.node(Op.custom("fused::swiglu"), [gt, up], [(act, (R, Fl))], {}, p + "swiglu")[0]
        dn = _linear(b, s, W, "d", R, D, fmt, act, p + "down_proj")
        if t > 1:
            dn = b.node(Op.custom("fused::all_reduce"), [dn], [(act, (R, D))], {}, p + "down_allreduce")[0]
        h = b.node(Op("add"), [h2, dn], [(act, (R, D))], {}, p + "ffn_residual")[0]
    hd.hidden_out = h
    if head == "none":
        hd.out = h
    else:
        Rh = R
        if last_token:
            h = b.node(Op.custom("fused::last_token"), [h], [(act, (batch, D))], {"tokens_per_seq": seq},
                       "last_token")[0]
            Rh = batch
        hf = b.node(Op.custom("fused::rms_norm"), [h, hd.final_norm], [(act, (Rh, D))],
                    {"eps": float(shape.eps)}, "final_norm_op")[0]
        W = {"wlm": hd.lm_w, "slm": hd.lm_s}
        logits = _linear(b, hf, W, "lm", Rh, Vr, lm_fmt or fmt, act, "lm_head")
        if head == "logits":
            hd.out = logits
        elif vpar:
            hd.out = b.node(Op.custom("fused::vocab_argmax"), [logits], [(I32, (Rh,))],
                            {"vocab_offset": v0}, "vocab_argmax")[0]
        else:
            hd.out = b.node(Op.custom("fused::argmax"), [logits], [(I32, (Rh,))], {}, "argmax")[0]
    b.output(hd.out)
    return b.build(), hd


# Matrices split by output feature (column-parallel) and by input feature
# (row-parallel) in the tensor-parallel layout; everything else is replicated.
_COLUMN_PARALLEL = ("q", "k", "v", "g", "u")
_ROW_PARALLEL = ("o", "d")


def shard_layer(full: dict, shape: DecoderShape, fmt: str, rank: int, world: int) -> dict:
    """One rank's slice of one layer's full (unsharded) weights.

    ``full`` maps the names of ``weight_shapes(shape, fmt, 1)`` (and
    ``k_cache`` / ``v_cache``) to numpy arrays in the graph's layouts: int4
    codes [N, K/2] with bf16 scales [N, K/32], int8 codes [N, K] with f32
    scales [N], MX codes [N, K] (E4M3) or [N, K/2] (E2M1, two per byte) with
    E8M0 scales [N, K/32], or plain [N, K] weights.  Column-parallel matrices keep rows
    [r*N/t, (r+1)*N/t); row-parallel ones keep columns [r*K/t, (r+1)*K/t) of
    the codes and the matching scale groups (per-channel int8 scales belong
    to the unsharded output rows and are kept whole).  The FFN dimension
    (gate/up rows, down_proj columns) follows ``ffn_shard`` in the format's
    ``ffn_unit`` instead.  KV caches, contiguous [batch, kv_heads, max_len,
    head_dim] or page pools [pages, kv_heads, page_size, head_dim], keep
    their rank's kv heads (the block table is the same on every rank).
    """
    t, r = world, rank
    f0, fn = ffn_shard(shape.ffn, t, r, ffn_unit(fmt))
    out = {}
    for name, arr in full.items():
        if name in ("attn_norm", "ffn_norm"):
            out[name] = arr
        elif name in ("k_cache", "v_cache"):
            g = arr.shape[1] // t
            out[name] = arr[:, r * g:(r + 1) * g].copy()
        else:
            kind, key = name[0], name[1:]
            if key in _COLUMN_PARALLEL:
                if key in ("g", "u"):
                    out[name] = arr[f0:f0 + fn].copy()
                else:
                    n = arr.shape[0] // t
                    out[name] = arr[r * n:(r + 1) * n].copy()
            elif key in _ROW_PARALLEL:
                if kind == "s" and fmt == "w8pc":
                    out[name] = arr  # per output channel: unsharded rows
                elif key == "d":
                    per = arr.shape[1] / shape.ffn  # array columns per feature: 1/2 codes, 1/32 scales, 1
                    out[name] = arr[:, int(f0 * per):int((f0 + fn) * per)].copy()
                else:
                    c = arr.shape[1] // t
                    out[name] = arr[:, r * c:(r + 1) * c].copy()
            else:
                raise ValueError(f"unknown weight {name}")
    return out
