"""The C-ABI library on a machine without a GPU: it builds, loads, exports
every entry point include/qwen3fused.h declares, agrees with the Python
binding on the argument struct, and rejects bad arguments on the host before
touching the device."""

import ctypes
import os
import re

import pytest

from tinyserver_b200 import _capi

HEADER_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_functions() -> set[str]:
    names = set()
    for f in os.listdir(HEADER_DIR):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(HEADER_DIR, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(qf_\w+)\s*\(", text, flags=re.M))
    return names


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for required in ("qf_kv_store_batched", "qf_kv_store_seq", "qf_rmsnorm", "qf_add_rmsnorm",
                     "qf_rope_cos_sin", "qf_qk_norm_rope_store", "qf_silu_and_mul",
                     "qf_embedding", "qf_build_slot_mapping", "qf_paged_attention_decode",
                     "qf_paged_attention_workspace_bytes", "qf_varlen_attention",
                     "qf_sample_tokens", "qf_uniforms_from_seeds", "qf_read_status"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for name in sorted(declared_functions()):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _capi.SIGNATURES, f"{name} has no ctypes signature in _capi"


def test_struct_abi_matches():
    lib = _capi.lib()
    assert lib.qf_qk_norm_rope_args_size() == ctypes.sizeof(_capi.QkNormRopeArgs)
    assert lib.qf_paged_attention_args_size() == ctypes.sizeof(_capi.PagedAttentionArgs)
    assert lib.qf_varlen_attention_args_size() == ctypes.sizeof(_capi.VarlenAttentionArgs)
    assert lib.qf_sample_args_size() == ctypes.sizeof(_capi.SampleArgs)


def test_version():
    assert _capi.lib().qf_version().decode().startswith("qwen3fused")


def test_host_side_argument_checks_return_before_any_launch():
    lib = _capi.lib()
    # negative sizes / unknown dtype / null pointers: rejected on the host
    assert lib.qf_silu_and_mul(None, 0, None, 0, None, 0, -1, 8, 2, None) == _capi.QF_ERR_INVALID
    assert lib.qf_silu_and_mul(None, 0, None, 0, None, 0, 4, 8, 2, None) == _capi.QF_ERR_INVALID
    assert lib.qf_rmsnorm(None, 0, None, None, 0, 4, 8, 1e-6, 9, None) == _capi.QF_ERR_INVALID
    assert lib.qf_embedding(None, 7, None, 1, 1, None, 1, 1, 1, 2, None, None) == \
        _capi.QF_ERR_INVALID
    a = _capi.QkNormRopeArgs()
    a.num_tokens, a.num_q_heads, a.num_kv_heads, a.head_dim, a.dtype = 4, 2, 1, 96, 2
    assert lib.qf_qk_norm_rope_store(ctypes.byref(a), None) == _capi.QF_ERR_UNSUPPORTED
    st = _capi.i64_array([0, 0, 0])
    ct = _capi.i64_array([0, 0, 0, 0])
    assert lib.qf_kv_store_batched(None, st, None, st, None, ct, None, ct, None, None, 1, 4, 2,
                                   8, 2, 0, 2, None, None) == _capi.QF_ERR_INVALID
    sa = _capi.SampleArgs()
    sa.batch, sa.vocab, sa.dtype = 2, 0, 2
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID  # empty vocab
    sa.vocab = 16
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID  # null pointers
    assert lib.qf_uniforms_from_seeds(None, None, -1, None, None) == _capi.QF_ERR_INVALID
    # zero-sized work is a no-op that needs no device
    sa.batch = 0
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_OK
    assert lib.qf_uniforms_from_seeds(None, None, 0, None, None) == _capi.QF_OK
    assert lib.qf_silu_and_mul(None, 0, None, 0, None, 0, 0, 8, 2, None) == _capi.QF_OK
    assert lib.qf_kv_store_seq(0, None, 0, 1, None, st, None, st, None, ct, None, ct, 0, 2, 8,
                               2, 4, 2, None, None) == _capi.QF_OK


def test_sampler_path_and_workspace_are_checked_on_the_host():
    """An unknown path, or the batch-wide path without a large enough,
    256-byte aligned workspace, is refused before any device work; the
    workspace size grows with the batch and is 0 for an empty one."""
    lib = _capi.lib()
    fake = 1 << 20  # never dereferenced: every call below returns on the host
    sa = _capi.SampleArgs()
    sa.logits, sa.logits_row_stride, sa.batch, sa.vocab, sa.dtype = fake, 16, 256, 16, 2
    sa.temperature = sa.top_k = sa.top_p = sa.uniforms = sa.out = fake
    sa.top_k_type = _capi.QF_I64
    sa.path = 7
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID
    sa.path = 2  # batch-wide, no workspace
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID
    need = lib.qf_sample_workspace_bytes(256)
    sa.workspace, sa.workspace_bytes = fake, need - 1
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID
    sa.workspace, sa.workspace_bytes = fake + 16, need  # misaligned
    assert lib.qf_sample_tokens(ctypes.byref(sa), None) == _capi.QF_ERR_INVALID
    assert lib.qf_sample_workspace_bytes(0) == 0
    assert 0 < lib.qf_sample_workspace_bytes(1) < need < 2 * lib.qf_sample_workspace_bytes(128) + 4096


def test_sampler_path_name_is_checked():
    import torch
    from tinyserver_b200.kernels import sampling
    z = torch.zeros(2, 4)
    with pytest.raises(ValueError, match="path must be one of"):
        sampling._launch(z, torch.ones(2), torch.zeros(2, dtype=torch.int64), torch.ones(2),
                         torch.zeros(2), None, None, "sample_tokens", "fastest")


def test_ensure_built_is_idempotent():
    p1 = _capi.ensure_built()
    mtime = os.path.getmtime(p1)
    assert _capi.ensure_built() == p1
    assert os.path.getmtime(p1) == mtime


@pytest.mark.parametrize("rc,exc", [(1, ValueError), (2, ValueError), (3, RuntimeError)])
def test_return_codes_map_to_exceptions(rc, exc):
    with pytest.raises(exc):
        _capi.check(rc, "op")
