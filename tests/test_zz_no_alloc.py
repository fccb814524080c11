"""The allocation-free decode attention entry point against the regular one.

Some callers cannot call cudaMalloc -- code running under stream capture in a
mode that refuses allocation, or a runtime that owns all device memory through
its own pool -- so strata_b200_attention_decode_bf16_noalloc keeps its split-KV
partials in a scratch area inside the library.  This file is named so pytest
collects it last; it also passes when run alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as ora
from tests.conftest import LIB
from tests.helpers import TOL_BF16, assert_close

pytestmark = pytest.mark.gpu

P, I64 = C.c_void_p, C.c_int64


def test_noalloc_attention_matches_the_scratch_taking_entry_point(cuda):
    torch = cuda
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

    batch, heads, kv_heads, d, max_len, fill = 4, 32, 8, 128, 2112, 2048

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(ora.to_bf16(a).view(np.int16))).cuda()

    kc = dev(ora.normal(31, (batch, kv_heads, max_len, d)))
    vc = dev(ora.normal(32, (batch, kv_heads, max_len, d)))
    q = dev(ora.normal(33, (batch, heads * d)))
    kn = dev(ora.normal(34, (batch, kv_heads * d)))
    vn = dev(ora.normal(35, (batch, kv_heads * d)))
    pos = torch.tensor([fill, fill - 3, 700, 5], dtype=torch.int32, device="cuda")
    kc2, vc2 = kc.clone(), vc.clone()
    scratch = torch.empty((lib.strata_b200_attention_decode_scratch_bytes(batch, heads, d, max_len),),
                          dtype=torch.uint8, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: C.c_void_p(t.data_ptr())

    for call in range(2):  # the shared scratch keeps the previous call's contents
        out_ref = torch.empty((batch, heads * d), dtype=torch.int16, device="cuda")
        out_na = torch.full((batch, heads * d), 0x7FC0, dtype=torch.int16, device="cuda")
        assert ref(ptr(q), ptr(kn), ptr(vn), ptr(kc), ptr(vc), ptr(pos), batch, heads, kv_heads, d, max_len,
                   ptr(scratch), ptr(out_ref), s) == 0
        assert noalloc(ptr(q), ptr(kn), ptr(vn), ptr(kc2), ptr(vc2), ptr(pos), batch, heads, kv_heads, d,
                       max_len, ptr(out_na), s) == 0
        torch.cuda.synchronize()
        got = ora.from_bf16(out_na.cpu().numpy().view(np.uint16))
        want = ora.from_bf16(out_ref.cpu().numpy().view(np.uint16))
        assert_close(got, want, TOL_BF16, f"no-alloc attention, call {call}")
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)

    # A shape that needs more scratch than the library holds is refused, not run.
    assert lib.strata_b200_noalloc_scratch_capacity() == 32 << 20
    big = 4096
    assert noalloc(ptr(q), ptr(kn), ptr(vn), ptr(kc), ptr(vc), ptr(pos), big, heads, kv_heads, d, 1 << 20,
                   ptr(out_ref), s) == -5
