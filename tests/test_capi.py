"""libdotl's C ABI on the host (no GPU): it loads, exports every symbol that
include/dotl.h declares, and rejects bad arguments with a status code and a
message before anything reaches a device."""

import ctypes
import os
import re

import pytest

from conftest import PKG, REPO

HEADER = os.path.join(REPO, "include", "dotl.h")
LIB = os.path.join(PKG, "lib", "libdotl.so")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        import kernel_ext

        kernel_ext.build()
    import dotl_ops

    return dotl_ops.load(LIB)


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(dotl_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = _declared()
    for n in ("dotl_linear", "dotl_attention", "dotl_layernorm", "dotl_identity_f32",
              "dotl_last_error", "dotl_device_error"):
        assert n in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version(lib):
    assert lib.dotl_abi_version() == 2


def _err(lib):
    return lib.dotl_last_error().decode()


def test_linear_rejects_unaligned_k(lib):
    rc = lib.dotl_linear(16, 4, 7, 7, 16, 16, 7, 16, 0, None, 0, None, 0, 16, 0, 16, 0, 1, None)
    assert rc == 2 and "multiples of 8" in _err(lib)


def test_linear_rejects_bad_modes(lib):
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 2, None, 0, None, 0, 16, 0, 16, 0, 1, None) == 1
    assert "act must be" in _err(lib)
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 0, None, 0, None, 9, 16, 0, 16, 0, 1, None) == 1
    assert "residual mode" in _err(lib)
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 0, None, 0, None, 0, 16, 5, 16, 0, 1, None) == 1
    assert "out dtype" in _err(lib)
    # operand and output codes: DOTL_F16 / DOTL_F16X2 only
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 0, None, 0, None, 0, 16, 0, 16, 0, 0, None) == 1
    assert "operands" in _err(lib)
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 0, None, 0, None, 0, 16, 3, 16, 0, 1, None) == 1
    assert "out dtype" in _err(lib)
    # masked residual needs the row mask
    assert lib.dotl_linear(16, 4, 8, 8, 16, 16, 8, 16, 0, 16, 16, None, 3, 16, 0, 16, 0, 1, None) == 1
    assert "row_valid" in _err(lib)


def test_linear_empty_m_is_ok(lib):
    assert lib.dotl_linear(None, 0, 8, 8, None, 16, 8, None, 0, None, 0, None, 0, None, 0, 16, 0, 1, None) == 0


def test_attention_rejects_head_dim(lib):
    st = (ctypes.c_int64 * 3)(0, 0, 0)
    for hd in (4, 12, 264):
        rc = lib.dotl_attention(16, 16, 16, 1, 1, 8, hd, st, st, st, None, 0, None, 0, 0.1, 16, 0, 1, None, 0, None)
        assert rc == 2 and "head_dim" in _err(lib)


def test_attention_rejects_generic_grid_overflow(lib):
    # head_dim 8 takes the CUDA-core kernel, one grid row per (batch, head)
    st = (ctypes.c_int64 * 3)(0, 0, 0)
    rc = lib.dotl_attention(16, 16, 16, 65536, 1, 8, 8, st, st, st, None, 0, None, 0, 0.1, 16, 0, 1, None, 0, None)
    assert rc == 2 and "65535" in _err(lib)


def test_attention_rejects_layout_and_mask(lib):
    st = (ctypes.c_int64 * 3)(0, 0, 0)
    assert lib.dotl_attention(16, 16, 16, 1, 1, 8, 64, st, st, st, None, 0, None, 0, 0.1, 16, 2, 1, None, 0, None) == 1
    assert "out_layout" in _err(lib)
    assert lib.dotl_attention(16, 16, 16, 1, 1, 8, 64, st, st, st, None, 1, None, 0, 0.1, 16, 0, 1, None, 0, None) == 1
    assert "needs mask" in _err(lib)
    assert lib.dotl_attention(16, 16, 16, 1, 1, 8, 64, st, st, st, None, 0, None, 0, 0.1, 16, 0, 0, None, 0, None) == 1
    assert "out dtype" in _err(lib)


def test_attention_rejects_unaligned_strides(lib):
    st = (ctypes.c_int64 * 3)(64 * 8, 64, 12)
    rc = lib.dotl_attention(16, 16, 16, 1, 1, 8, 64, st, st, st, None, 0, None, 0, 0.1, 16, 0, 1, None, 0, None)
    assert rc == 2 and "multiples of 8" in _err(lib)


def test_layernorm_rejects(lib):
    assert lib.dotl_layernorm(16, None, 16, 16, None, 16, 0, None, 4, 4096, 1e-5, None) == 2
    assert "2048" in _err(lib)
    assert lib.dotl_layernorm(16, 16, 16, 16, None, 16, 0, None, 4, 64, 1e-5, None) == 1
    assert "x_new" in _err(lib)
    assert lib.dotl_layernorm(16, None, 16, 16, None, 16, 7, None, 4, 64, 1e-5, None) == 1


def test_identity_rejects_negative(lib):
    assert lib.dotl_identity_f32(None, None, -1, None) == 1
    assert "negative" in _err(lib)
    assert lib.dotl_identity_f32(None, None, 0, None) == 0


def test_build_flags_target_sm100a():
    import kernel_ext

    cmd = " ".join(kernel_ext.build_command())
    assert "arch=compute_100a,code=sm_100a" in cmd and "-lineinfo" in cmd


def test_allreduce_ln_rejects(lib):
    P2 = ctypes.c_void_p * 2
    parts, sigs, outs = P2(16, 32), P2(48, 64), P2(80, 96)

    def call(world=2, rank=0, D=128, dtype=0, timeout=2000, p=parts, local=0, blocks=1, sig_bytes=68,
             status=None):
        return lib.dotl_allreduce_ln(world, rank, p, sigs, None, outs, dtype, 0, local, 16, None, None, 16, 16,
                                     1e-5, None, 8, D, blocks, sig_bytes, status, timeout, None)

    assert call(world=9) == 1 and "world" in _err(lib)
    assert call(rank=2) == 1 and "rank" in _err(lib)
    assert call(D=130) == 1 and "multiple of 4" in _err(lib)
    assert call(D=4096) == 1
    assert call(dtype=5) == 1 and "dtype" in _err(lib)
    assert call(timeout=0) == 1 and "timeout_ms" in _err(lib)
    assert call(p=P2(16, None)) == 1 and "NULL" in _err(lib)
    assert call(p=P2(16, 40)) == 1 and "aligned" in _err(lib)
    assert call(local=1) == 1 and "push" in _err(lib)
    # signal areas sized for one grid, called with another: rejected before launch
    assert call(blocks=2) == 1 and "signal areas" in _err(lib)
    assert call(sig_bytes=4096) == 1 and "signal areas" in _err(lib)
    assert call(status=6) == 1 and "status" in _err(lib)


def test_linear_peer_rejects(lib):
    P2 = ctypes.c_void_p * 2
    outs = P2(256, 512)
    # M must be world x rows_per_rank with rows_per_rank a multiple of 128
    assert lib.dotl_linear_peer(16, 300, 64, 64, 16, 64, 64, None, 2, outs, 150, 64, None) == 2
    assert "rows_per_rank" in _err(lib)
    assert lib.dotl_linear_peer(16, 256, 64, 64, 16, 64, 64, None, 9, outs, 128, 64, None) == 1
    assert lib.dotl_linear_peer(16, 256, 60, 64, 16, 64, 64, None, 2, outs, 128, 64, None) == 2


def test_peer_setup_rejects_and_sizes(lib):
    n = ctypes.c_int64(0)
    assert lib.dotl_peer_signal_bytes(296, ctypes.byref(n)) == 0 and n.value == 296 * 17 * 4
    assert lib.dotl_peer_signal_bytes(0, ctypes.byref(n)) == 1
    p = ctypes.c_void_p(0)
    assert lib.dotl_peer_alloc(0, ctypes.byref(p)) == 1
    assert lib.dotl_ipc_open(None, ctypes.byref(p)) == 1
    assert lib.dotl_peer_free(None) == 0 and lib.dotl_ipc_close(None) == 0


def test_ffn_rejects(lib):
    def call(D=256, F=1024, lda=256, mode=0, resid=None, rv=None, normed=64, dtype=1, eps=1e-5, x_out=None):
        return lib.dotl_ffn(64, 100, D, lda, 64, F, D, 64, 64, F, 64, resid, D, rv, mode, x_out, D, 64, 64,
                            eps, normed, dtype, D, None, None)

    assert call(D=192) == 2 and "128 or 256" in _err(lib)
    assert call(F=1000) == 2 and "multiple of 128" in _err(lib)
    assert call(mode=4) == 1 and "residual mode" in _err(lib)
    assert call(mode=1) == 1 and "needs resid" in _err(lib)
    assert call(mode=3, resid=64) == 1 and "row_valid" in _err(lib)
    assert call(dtype=7) == 1 and "dtype" in _err(lib)
    assert call(eps=-1.0) == 1 and "eps" in _err(lib)
    assert call(lda=100) == 2 and "multiples of 8" in _err(lib)
    assert call(normed=None) == 1 and "NULL" in _err(lib)
    assert call(x_out=72) == 2 and "x_out" in _err(lib)
    assert lib.dotl_ffn(None, 0, 256, 256, None, 1024, 256, None, None, 1024, None, None, 256, None, 0,
                        None, 256, None, None, 1e-5, None, 1, 256, None, None) == 0   # M = 0: nothing to do


def _prototypes():
    """name -> parameter declarations, from include/dotl.h."""
    text = re.sub(r"/\*.*?\*/", " ", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int|const char\s*\*)\s*(dotl_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
    return out


def _kind_of_decl(decl):
    if "*" in decl:
        return "ptr"
    if "int64_t" in decl:
        return "i64"
    if "float" in decl:
        return "f32"
    if "int" in decl:
        return "i32"
    raise AssertionError(f"unclassified parameter {decl!r}")


def _kind_of_ctype(t):
    if t in (ctypes.c_void_p, ctypes.c_char_p) or hasattr(t, "_type_") and isinstance(t._type_, type):
        return "ptr"
    return {ctypes.c_int64: "i64", ctypes.c_float: "f32", ctypes.c_int: "i32", ctypes.c_uint: "i32"}[t]


def test_ctypes_signatures_match_the_header():
    """Every binding dotl_ops declares has the header's parameter count and
    kinds (pointer, int64, int, float): a drifted ctypes signature would pass
    arguments in the wrong registers without any error."""
    import dotl_ops

    protos = _prototypes()
    assert set(dotl_ops._SIGNATURES) <= set(protos), set(dotl_ops._SIGNATURES) - set(protos)
    for name, (argtypes, _restype) in dotl_ops._SIGNATURES.items():
        want = [_kind_of_decl(d) for d in protos[name]]
        got = [_kind_of_ctype(t) for t in argtypes]
        assert got == want, f"{name}: ctypes {got} != header {want}"
