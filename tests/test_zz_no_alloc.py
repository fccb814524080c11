"""The allocation-free decode attention entry point.

Some callers cannot call cudaMalloc: code running while a stream is captured
in a mode that refuses allocation, or a runtime whose device memory all
belongs to its own pool.  strata_b200_attention_decode_bf16_noalloc serves
them by keeping its split-KV partials in a scratch array inside the library
instead of a buffer the caller passes.

Only the CUDA-core kernel writes partials; it runs when a kv head serves more
than 8 query heads (here 32 query heads over 2 kv heads).  The first test
uses that shape with a long cache, so every call goes through the library's
scratch array; it checks two calls in a row (the array keeps the previous
call's contents) against the oracle and against the scratch-taking entry
point.  The second test checks that a shape the tensor-core kernel runs
needs no scratch and is therefore not refused however large it is.

This file is named so that pytest collects it last; it also passes when run
alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as ora
from tests.conftest import LIB
from tests.helpers import TOL_BF16, assert_close

pytestmark = pytest.mark.gpu

P, I64 = C.c_void_p, C.c_int64


def _entry_points():
    lib = C.CDLL(LIB)
    ref = lib.strata_b200_attention_decode_bf16
    ref.argtypes = [P, P, P, P, P, P, I64, I64, I64, I64, I64, P, P, P]
    ref.restype = C.c_int32
    noalloc = lib.strata_b200_attention_decode_bf16_noalloc
    noalloc.argtypes = [P, P, P, P, P, P, I64, I64, I64, I64, I64, P, P]
    noalloc.restype = C.c_int32
    lib.strata_b200_attention_decode_scratch_bytes.argtypes = [I64, I64, I64, I64]
    lib.strata_b200_attention_decode_scratch_bytes.restype = C.c_uint64
    lib.strata_b200_noalloc_scratch_capacity.restype = C.c_uint64
    return lib, ref, noalloc


def _run_calls(torch, shape, positions, seed):
    """Run the regular and the allocation-free entry points on the same
    inputs, once per entry of `positions`, and check both against the oracle
    (KV append at pos, then attention over 0..pos)."""
    lib, ref, noalloc = _entry_points()
    batch, heads, kv_heads, d, max_len, fill = shape

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(ora.to_bf16(a).view(np.int16))).cuda()

    kc_h = ora.round_bf16(ora.normal(seed, (batch, kv_heads, max_len, d)))
    vc_h = ora.round_bf16(ora.normal(seed + 1, (batch, kv_heads, max_len, d)))
    kc_h[:, :, fill:] = 0.0
    vc_h[:, :, fill:] = 0.0
    kc, vc = dev(kc_h), dev(vc_h)
    kc2, vc2 = kc.clone(), vc.clone()
    scratch = torch.empty((max(1, lib.strata_b200_attention_decode_scratch_bytes(batch, heads, d, max_len)),),
                          dtype=torch.uint8, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: C.c_void_p(t.data_ptr())
    errs = []
    for call, pos_l in enumerate(positions):
        q_h = ora.round_bf16(ora.normal(seed + 10 + 3 * call, (batch, heads * d)))
        kn_h = ora.round_bf16(ora.normal(seed + 11 + 3 * call, (batch, kv_heads * d)))
        vn_h = ora.round_bf16(ora.normal(seed + 12 + 3 * call, (batch, kv_heads * d)))
        q, kn, vn = dev(q_h), dev(kn_h), dev(vn_h)
        pos_np = np.array(pos_l, np.int32)
        pos = torch.from_numpy(pos_np).cuda()
        out_ref = torch.empty((batch, heads * d), dtype=torch.int16, device="cuda")
        out_na = torch.full((batch, heads * d), 0x7FC0, dtype=torch.int16, device="cuda")  # NaN fill
        assert ref(ptr(q), ptr(kn), ptr(vn), ptr(kc), ptr(vc), ptr(pos), batch, heads, kv_heads, d, max_len,
                   ptr(scratch), ptr(out_ref), s) == 0
        assert noalloc(ptr(q), ptr(kn), ptr(vn), ptr(kc2), ptr(vc2), ptr(pos), batch, heads, kv_heads, d,
                       max_len, ptr(out_na), s) == 0
        torch.cuda.synchronize()
        for b in range(batch):  # the oracle's cache after this call's append
            kc_h[b, :, pos_np[b]] = kn_h[b].reshape(kv_heads, d)
            vc_h[b, :, pos_np[b]] = vn_h[b].reshape(kv_heads, d)
        want = ora.attention(q_h, kc_h, vc_h, np.arange(batch), pos_np, heads, kv_heads, d,
                             threads=ora.max_threads())
        got = ora.from_bf16(out_na.cpu().numpy().view(np.uint16))
        errs.append(assert_close(got, want, TOL_BF16, f"allocation-free attention vs oracle, call {call}"))
        got_ref = ora.from_bf16(out_ref.cpu().numpy().view(np.uint16))
        assert_close(got, got_ref, TOL_BF16, f"allocation-free vs regular entry point, call {call}")
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    return errs


def test_noalloc_attention_uses_its_scratch_and_matches_the_oracle(cuda):
    """16 query heads per kv head: the CUDA-core kernel with split-KV partials
    in the library's scratch array (33 splits of 64 positions); two calls in
    a row with different positions and appended rows."""
    torch = cuda
    lib, _, _ = _entry_points()
    shape = batch, heads, kv_heads, d, max_len, fill = 4, 32, 2, 128, 2112, 2048
    assert lib.strata_b200_noalloc_scratch_capacity() == 32 << 20
    _run_calls(torch, shape, [[fill, fill - 3, 700, 5], [fill - 1, 129, 2000, 64]], seed=31)


def test_noalloc_sizes_its_scratch_by_the_kernel_that_runs(cuda):
    """A shape on the tensor-core kernel (8 query heads per kv head or fewer)
    merges its splits on chip and needs no scratch, so the allocation-free
    entry point runs it at any size; a wide-group shape whose partials do not
    fit the scratch array is refused before anything is launched."""
    torch = cuda
    _, _, noalloc = _entry_points()
    # 64 x 32 heads over 4160 positions: 35 MB of partials under the old
    # worst-case sizing, none on the tensor-core kernel.
    _run_calls(torch, (64, 32, 8, 128, 4160, 4096), [[4096 - (i % 7) for i in range(64)]], seed=41)
    # 16 query heads per kv head, 64 sequences over 65536 positions: 545 MB of
    # partials, more than the 32 MiB array -- STRATA_RESOURCE_EXHAUSTED.
    t = torch.zeros(16, dtype=torch.int16, device="cuda")
    p = C.c_void_p(t.data_ptr())
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert noalloc(p, p, p, p, p, p, 64, 32, 2, 128, 1 << 16, p, s) == -5
