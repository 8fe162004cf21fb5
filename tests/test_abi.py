"""The C-ABI library loads, exports every symbol include/lizard_cuda.h declares,
and rejects bad arguments with an error code and message. No GPU needed: every
call here fails validation before any CUDA call."""
import ctypes
import inspect
import re

import pytest
import torch

from conftest import ROOT


def declared_symbols():
    text = (ROOT / "include" / "lizard_cuda.h").read_text()
    return sorted(set(re.findall(r"\b(lz_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib(built_lib):
    from lizard_cuda import _lib
    return _lib.load()


def test_header_declares_the_expected_entry_points():
    syms = declared_symbols()
    for name in ("lz_gla_fwd", "lz_gla_bwd", "lz_swa_fwd", "lz_swa_bwd", "lz_abi_version",
                 "lz_last_error_string", "lz_gla_saved_bytes", "lz_swa_bwd_workspace_bytes"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_hedgehog_rows_max_switch_round_trips(lib):
    assert lib.lz_hedgehog_set_rows_max(100) == -1
    assert lib.lz_hedgehog_set_rows_max(-5) == 100
    assert lib.lz_hedgehog_set_rows_max(-1) == -1


def test_abi_version(lib):
    from lizard_cuda import _lib
    assert lib.lz_abi_version() == _lib.ABI_VERSION == 3


def test_buffer_size_queries(lib):
    B, H, L, F, D = 2, 3, 150, 24, 20
    nt = -(-L // 64)
    saved = lib.lz_gla_saved_bytes(B, H, L, F, D, 64)
    assert saved >= B * H * L * D * 4 + 2 * B * H * L * 4 + B * H * nt * F * (2 * D + 4)
    assert lib.lz_gla_bwd_workspace_bytes(B, H, L, F, D, 64) >= B * H * nt * F * D * 2
    assert lib.lz_swa_saved_bytes(B, H, L, D) >= B * H * L * 4 * (1 + D)
    assert lib.lz_swa_bwd_workspace_bytes(B, H, L, D, 4) >= B * H * L * 4
    assert lib.lz_gla_saved_bytes(0, H, L, F, D, 64) == 0


def _fake(n=1):
    # never dereferenced: validation rejects the calls first
    return [ctypes.c_void_p(0x1000 * (i + 1)) for i in range(n)]


def test_gqa_entries_validate_head_counts(lib):
    p = _fake(6)
    # H = 6 query heads over Hkv = 4 key/value heads does not divide
    rc = lib.lz_swa_fwd_gqa(*p[:3], None, None, None, 0, 16, p[3], None, 0, 1, 6, 4, 64, 64,
                            None)
    assert rc == 1 and b"divide" in lib.lz_last_error_string()
    rc = lib.lz_gla_fwd_gqa(*p[:4], 0, p[4], None, 0, None, 0, 1, 6, 4, 64, 64, 64, 64, None)
    assert rc == 1 and b"divide" in lib.lz_last_error_string()
    rc = lib.lz_gla_bwd_gqa(*p[:4], 0, p[4], 1 << 30, p[5], *_fake(3), 0, p[0], p[1], 1 << 30,
                            1, 6, 0, 64, 64, 64, 64, None)
    assert rc == 1 and b"divide" in lib.lz_last_error_string()
    # the grouped backward needs room for the per-head dfk / dv before the group sums
    plain = lib.lz_gla_bwd_workspace_bytes(2, 8, 256, 64, 64, 64)
    assert lib.lz_gla_bwd_gqa_workspace_bytes(2, 8, 8, 256, 64, 64, 64) == plain
    assert (lib.lz_gla_bwd_gqa_workspace_bytes(2, 8, 2, 256, 64, 64, 64)
            >= plain + 2 * 8 * 256 * (64 + 64) * 4)
    assert lib.lz_gla_bwd_gqa_workspace_bytes(2, 8, 3, 256, 64, 64, 64) == 0


def test_forward_workspace_plans_shared_states(lib):
    # F = 256 runs the chunk-parallel schedule; without a saved buffer and with a
    # gate shared by the heads, its states are per key/value head
    B, H, Hkv, L, F, D = 4, 32, 8, 1024, 256, 64
    per_q = lib.lz_gla_fwd_gqa_workspace_bytes(B, H, Hkv, L, F, D, 64, 0, 1)
    shared = lib.lz_gla_fwd_gqa_workspace_bytes(B, H, Hkv, L, F, D, 64, 0, 0)
    assert per_q == lib.lz_gla_fwd_workspace_bytes(B, H, L, F, D, 64) > 0
    assert per_q >= 4 * (shared - 4096) and shared >= B * Hkv * (L // 64) * F * D * 4
    assert lib.lz_gla_fwd_gqa_workspace_bytes(B, H, Hkv, L, F, D, 64, 1, 0) == per_q
    assert lib.lz_gla_fwd_gqa_workspace_bytes(B, H, 3, L, F, D, 64, 0, 0) == 0


def test_rope_entries_validate(lib):
    p = _fake(4)
    # odd head dim cannot be rotated in halves
    rc = lib.lz_rope_split(p[0], 0, 0, 0, 0, p[1], p[2], 0, 0, 0, p[3], None, 1, 1, 8, 63, None)
    assert rc == 1 and b"even" in lib.lz_last_error_string()
    rc = lib.lz_rope_split(p[0], 7, 0, 0, 0, p[1], p[2], 0, 0, 0, p[3], None, 1, 1, 8, 64, None)
    assert rc == 1 and b"dtype" in lib.lz_last_error_string()
    rc = lib.lz_rope_bwd(p[0], p[1], p[2], 5, 0, 0, p[3], 0, 1, 1, 8, 64, None)
    assert rc == 1 and b"cos" in lib.lz_last_error_string()
    rc = lib.lz_rope_bwd(None, p[1], p[2], 0, 0, 0, p[3], 0, 1, 1, 8, 64, None)
    assert rc == 1


def test_decode_entries_validate(lib):
    p = _fake(8)
    # state heads must be H, or Hkv with a shared gate
    rc = lib.lz_gla_decode(*p[:4], 1, p[4], p[5], p[6], 2, 8, 2, 2, 64, 64, None)
    assert rc == 1 and b"state heads" in lib.lz_last_error_string()
    rc = lib.lz_gla_decode(*p[:4], 0, p[4], p[5], p[6], 2, 8, 2, 2, 300, 64, None)
    assert rc == 2
    rc = lib.lz_gla_decode(*p[:4], 0, p[4], p[5], p[6], 2, 6, 2, 2, 64, 64, None)
    assert rc == 2 and b"query heads per state" in lib.lz_last_error_string()
    rc = lib.lz_swa_decode(*p[:3], 0, 0, 0, 0, 0, 0, 0, p[3], p[4], 0, 0, p[5], p[6], p[7],
                           None, 0, p[0], 1, 4, 3, 16, 64, None)
    assert rc == 1 and b"divide" in lib.lz_last_error_string()
    rc = lib.lz_swa_decode(*p[:3], 0, 0, 0, 0, 0, 0, 0, p[3], p[4], 0, 0, p[5], p[6], p[7],
                           None, 0, p[0], 1, 4, 2, 16, 63, None)
    assert rc == 1 and b"even" in lib.lz_last_error_string()


def test_gla_fwd_rejects_null_pointers(lib):
    rc = lib.lz_gla_fwd(None, None, None, None, 0, None, None, 0, None, 0, 1, 1, 8, 8, 8, 64, None)
    assert rc == 1
    assert b"null" in lib.lz_last_error_string()


def test_gla_fwd_rejects_bad_sizes(lib):
    p = _fake(5)
    assert lib.lz_gla_fwd(*p[:4], 0, p[4], None, 0, None, 0, 0, 1, 8, 8, 8, 64, None) == 1
    assert lib.lz_gla_fwd(*p[:4], 0, p[4], None, 0, None, 0, 1, 1, 8, 8, 8, 0, None) == 1
    assert lib.lz_gla_fwd(*p[:4], 0, p[4], None, 0, None, 0, 1, 1, 8, 300, 8, 64, None) == 2
    assert b"feature dim" in lib.lz_last_error_string()


def test_gla_fwd_rejects_small_saved_buffer(lib):
    p = _fake(6)
    rc = lib.lz_gla_fwd(*p[:4], 0, p[4], p[5], 16, None, 0, 1, 1, 8, 8, 8, 64, None)
    assert rc == 4
    assert b"saved" in lib.lz_last_error_string()


def test_schedule_setting_and_forward_workspace(lib):
    # one chunk: both schedules are the same work, the walk is planned
    assert lib.lz_gla_fwd_workspace_bytes(1, 32, 64, 64, 64, 64) == 0
    # 32 heads of 2048 tokens: too few chains for a walk, chunk-parallel planned
    auto = lib.lz_gla_fwd_workspace_bytes(1, 32, 2048, 64, 64, 64)
    assert auto >= 32 * 32 * 64 * 64 * 4
    # many heads: the walk
    assert lib.lz_gla_fwd_workspace_bytes(8, 32, 2048, 128, 128, 64) == 0
    assert lib.lz_gla_set_schedule(1) == 0
    try:
        assert lib.lz_gla_fwd_workspace_bytes(1, 32, 2048, 64, 64, 64) == 0
        walk_bwd = lib.lz_gla_bwd_workspace_bytes(1, 32, 2048, 64, 64, 64)
        assert lib.lz_gla_set_schedule(2) == 1
        assert lib.lz_gla_fwd_workspace_bytes(8, 32, 2048, 128, 128, 64) > 0
        assert lib.lz_gla_bwd_workspace_bytes(1, 32, 2048, 64, 64, 64) > walk_bwd
        assert lib.lz_gla_set_schedule(7) == -1
        assert b"schedule" in lib.lz_last_error_string()
        assert lib.lz_gla_set_schedule(2) == 2
    finally:
        lib.lz_gla_set_schedule(0)


def test_f128_schedule_crossover(lib):
    """At F = D = 128 the tensor-core walk runs one chain's time whatever the
    head count; the chunk-parallel schedule (which needs a forward workspace and
    a larger backward one) is planned only for 20 heads or fewer, the measured
    crossover at L = 2048 ... 16384."""
    for L in (2048, 16384):
        assert lib.lz_gla_fwd_workspace_bytes(1, 20, L, 128, 128, 64) > 0
        assert lib.lz_gla_fwd_workspace_bytes(1, 21, L, 128, 128, 64) == 0
        assert lib.lz_gla_fwd_workspace_bytes(1, 32, L, 128, 128, 64) == 0
        split_bwd = lib.lz_gla_bwd_workspace_bytes(1, 20, L, 128, 128, 64)
        walk_bwd = lib.lz_gla_bwd_workspace_bytes(1, 21, L, 128, 128, 64)
        # per head, the chunk-parallel backward also keeps the fp32 increments
        assert split_bwd / 20 > walk_bwd / 21


def test_gla_fwd_rejects_missing_workspace(lib):
    p = _fake(5)
    rc = lib.lz_gla_fwd(*p[:4], 0, p[4], None, 0, None, 0, 1, 32, 2048, 64, 64, 64, None)
    assert rc == 4
    assert b"workspace" in lib.lz_last_error_string()


def test_gla_bwd_rejects_bad_grad_dtype(lib):
    p = _fake(12)
    rc = lib.lz_gla_bwd(*p[:4], 0, p[4], 1 << 30, p[5], p[6], p[7], p[8], 7, p[9], p[10],
                        1 << 30, 1, 1, 8, 8, 8, 64, None)
    assert rc == 1
    assert b"grad_dtype" in lib.lz_last_error_string()


def test_swa_rejects_bad_window_and_sinks(lib):
    p = _fake(6)
    assert lib.lz_swa_fwd(*p[:3], None, None, None, 0, 0, p[4], None, 0, 1, 1, 8, 8, None) == 1
    assert b"window" in lib.lz_last_error_string()
    assert lib.lz_swa_fwd(*p[:3], None, None, None, 2, 4, p[4], None, 0, 1, 1, 8, 8, None) == 1
    assert lib.lz_swa_fwd(*p[:3], None, None, p[3], 33, 4, p[4], None, 0, 1, 1, 8, 8, None) == 2
    assert lib.lz_swa_fwd(*p[:3], None, None, p[3], 1, 4, p[4], None, 0, 1, 1, 8, 256, None) == 2
    assert lib.lz_swa_fwd(*p[:3], p[5], None, p[3], 1, 4, p[4], None, 0, 1, 1, 8, 8, None) == 1
    assert b"q_lo" in lib.lz_last_error_string()


def test_error_string_is_cleared_by_a_new_call(lib):
    lib.lz_gla_fwd(None, None, None, None, 0, None, None, 0, None, 0, 1, 1, 8, 8, 8, 64, None)
    assert lib.lz_last_error_string() != b""
    lib.lz_abi_version()
    p = _fake(5)
    lib.lz_swa_fwd(*p[:3], None, None, None, 0, 0, p[4], None, 0, 1, 1, 8, 8, None)
    assert b"window" in lib.lz_last_error_string()


def test_python_signatures_match_the_reference(built_lib):
    import lizard_cuda
    sig = inspect.signature(lizard_cuda.gla)
    assert list(sig.parameters) == ["fq", "fk", "v", "log_gamma", "chunk"]
    assert sig.parameters["chunk"].default == 64
    sig = inspect.signature(lizard_cuda.swa)
    assert list(sig.parameters) == ["q", "k", "v", "meta", "window", "fwd_blocks", "bwd_blocks"]
    assert lizard_cuda.swa.__defaults__ == ((64, 64), (64, 64))


def test_cpu_tensors_are_rejected_not_computed(built_lib):
    import lizard_cuda
    x = torch.rand(1, 1, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        lizard_cuda.gla(x, x, x, torch.zeros(1, 4))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        lizard_cuda.swa(x, x, x, torch.zeros(4), 4)


def test_layer_accepts_only_the_cuda_backend(built_lib):
    from types import SimpleNamespace

    from lizard_cuda.layer import LizardAttention
    cfg = SimpleNamespace(hidden_size=32, num_attention_heads=2, num_key_value_heads=1)
    layer = LizardAttention(cfg, 0, window=8, num_meta=2, feature_dim=4)
    names = sorted(n for n, _ in layer.named_parameters())
    assert names == sorted(["q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight",
                            "phi_q.weight", "phi_k.weight", "W_gamma.weight", "meta_tokens",
                            "alpha_blend"])
    with pytest.raises(ValueError, match="cuda backend only"):
        LizardAttention(cfg, 0, backend="torch")
