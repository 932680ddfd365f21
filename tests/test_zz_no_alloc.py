"""The allocation-free decode attention entry point, through the C ABI.

Some callers cannot allocate device memory: a host framework that passes this
library only raw pointers and owns every allocation, a runtime that reserves
all device memory at start, or a latency-bound loop that cannot take the
device synchronisation cudaMalloc implies.  qf_paged_attention_decode_noalloc
serves them from a fixed device array inside the library.  This test calls it
twice in a row and checks each result against the regular entry point
(qf_paged_attention_decode with a caller-provided workspace), within the
bf16 tolerance of tests/common.py, and checks that a call too large for the
array is refused before any device work.

The file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process.
"""

import ctypes
import math

import pytest
import torch

from tests.common import assert_close
from tinyserver_b200 import _capi
from tinyserver_b200._runtime import status_word, stream_ptr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _inputs(lens, hq=32, hkv=8, hd=128, bsz=16, seed=11):
    g = torch.Generator().manual_seed(seed)
    per = [max(1, -(-n // bsz)) for n in lens]
    nblk = sum(per) + 4
    q = torch.randn(len(lens), hq, hd, generator=g).to(torch.bfloat16)
    kc = torch.randn(nblk, hkv, bsz, hd, generator=g).to(torch.bfloat16)
    vc = torch.randn(nblk, hkv, bsz, hd, generator=g).to(torch.bfloat16)
    phys = torch.randperm(nblk, generator=g)[:sum(per)]
    bt = torch.zeros(len(lens), max(per), dtype=torch.int32)
    cur = 0
    for i, n in enumerate(per):
        bt[i, :n] = phys[cur:cur + n].to(torch.int32)
        cur += n
    return (q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV),
            torch.tensor(lens, dtype=torch.int32, device=DEV))


def _args(q, kc, vc, bt, sl, out, workspace=None):
    a = _capi.PagedAttentionArgs()
    a.q, a.q_stride_seq, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    for i in range(4):
        a.cache_strides[i] = kc.stride(i)
    a.num_blocks, a.block_size = kc.shape[0], kc.shape[2]
    a.block_tables, a.block_tables_row_stride = bt.data_ptr(), bt.stride(0)
    a.max_blocks_per_seq = bt.shape[1]
    a.seq_lens = sl.data_ptr()
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim = \
        q.shape[0], q.shape[1], kc.shape[1], q.shape[2]
    a.scale = 1.0 / math.sqrt(q.shape[2])
    a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    a.dtype = _capi.QF_BF16
    a.status = status_word(DEV).data_ptr()
    return a


def _flags():
    out = ctypes.c_int32(0)
    _capi.lib().qf_read_status(status_word(DEV).data_ptr(), ctypes.byref(out), 1,
                               stream_ptr(DEV))
    return out.value


def test_noalloc_matches_the_allocating_entry_point_twice():
    torch.cuda.set_device(DEV)
    lib = _capi.lib()
    q, kc, vc, bt, sl = _inputs([1, 17, 513, 1400, 3000, 4095])
    need = lib.qf_paged_attention_workspace_bytes(q.shape[0], q.shape[1], q.shape[2],
                                                  bt.shape[1] * kc.shape[2])
    assert 0 < need <= lib.qf_paged_attention_noalloc_capacity()
    ws = torch.empty(need // 4, dtype=torch.float32, device=DEV)
    expected = torch.empty_like(q)
    rc = lib.qf_paged_attention_decode(_args(q, kc, vc, bt, sl, expected, ws), stream_ptr(DEV))
    assert rc == _capi.QF_OK
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = lib.qf_paged_attention_decode_noalloc(_args(q, kc, vc, bt, sl, out),
                                                   stream_ptr(DEV))
        assert rc == _capi.QF_OK, f"call {call}: rc {rc}"
        torch.cuda.synchronize()
        assert_close(out, expected, f"no-alloc call {call}")
        # both entry points choose the same partitions on the same inputs, so
        # the outputs are bit-identical, not only within tolerance
        assert torch.equal(out, expected), f"no-alloc call {call} differs from the allocating one"
    assert _flags() == 0


def test_noalloc_refuses_a_call_larger_than_its_array():
    torch.cuda.set_device(DEV)
    lib = _capi.lib()
    q, kc, vc, bt, sl = _inputs([40])
    out = torch.empty_like(q)
    a = _args(q, kc, vc, bt, sl, out)
    # claim block tables long enough that the partials exceed the array; the
    # size check comes before any device work, so nothing is launched
    a.max_blocks_per_seq = 1 << 20
    cap = lib.qf_paged_attention_noalloc_capacity()
    assert lib.qf_paged_attention_workspace_bytes(1, 32, 128, (1 << 20) * 16) > cap
    assert lib.qf_paged_attention_decode_noalloc(a, stream_ptr(DEV)) == _capi.QF_ERR_SCRATCH
