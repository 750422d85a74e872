"""The C-ABI library loads, exports every entry point include/exl3_b200.h declares, and rejects bad arguments with
status codes before touching a GPU. CPU only: no compute call reaches a device."""
import os
import re

import pytest
import torch

from exl3_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "exl3_b200.h")).read()
    return sorted(set(re.findall(r"EXL3_API\s+[\w\s\*]*?\b(exl3_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    decl = declared_symbols()
    assert len(decl) >= 10
    for name in decl:
        assert hasattr(lib, name), name
    assert sorted(L.exported_symbols()) == decl


def declared_arities():
    """Parameter count of every EXL3_API declaration in the header (void parameter lists count 0)."""
    src = open(os.path.join(ROOT, "include", "exl3_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"EXL3_API\s+[\w\s\*]*?\b(exl3_\w+)\s*\(([^)]*)\)\s*;", src):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_prototypes_match_the_header():
    """Every ctypes prototype of the Python mirror has the header's number of parameters."""
    ar = declared_arities()
    assert set(ar) == set(declared_symbols())
    assert {n for n, _, _ in L._PROTOS} == set(ar), "every declared entry point has a prototype"
    for name, _, args in L._PROTOS:
        assert name in ar, name
        assert len(args) == ar[name], (name, len(args), ar[name])


def test_version_and_error_text():
    assert L.lib().exl3_version() >= 100
    assert isinstance(L.lib().exl3_last_error(), bytes)


def test_argument_validation_returns_status_codes():
    lib = L.lib()

    def gemv(x=16, M=1, packed=16, k=128, n=128, K=3, cb=2, ws=16, ws_bytes=1 << 30, groups=0):
        return lib.exl3_gemv(x, 0, k, M, packed, 16, 16, k, n, K, cb, 16, 0, n, ws, ws_bytes, groups, None)

    # codebook other than mul1
    assert gemv(cb=1) == L.EXL3_ERR_UNSUPPORTED
    assert b"mul1" in lib.exl3_last_error()
    # K out of range
    assert lib.exl3_dequant(16, 128, 128, 9, 2, 0, 128, 16, 128, None) == L.EXL3_ERR_UNSUPPORTED
    assert gemv(K=0) == L.EXL3_ERR_UNSUPPORTED
    # k not a multiple of 128
    assert gemv(k=100) == L.EXL3_ERR_ARG
    # too many rows per call (16 at most)
    assert gemv(M=17) == L.EXL3_ERR_ARG
    # the split-unit finisher wait: 0 .. 100 ms (host-side setting, no device involved)
    assert lib.exl3_set_finisher_wait(100_000_001) == L.EXL3_ERR_ARG
    assert lib.exl3_set_finisher_wait(0) == L.EXL3_OK
    assert lib.exl3_set_finisher_wait(20000) == L.EXL3_OK
    # misaligned packed weights
    assert gemv(packed=18) == L.EXL3_ERR_ARG
    # workspace missing or too small
    assert gemv(ws=0) == L.EXL3_ERR_WORKSPACE
    assert gemv(ws_bytes=16) == L.EXL3_ERR_WORKSPACE
    # dequant slice outside the matrix
    assert lib.exl3_dequant(16, 128, 128, 3, 2, 64, 128, 16, 128, None) == L.EXL3_ERR_ARG
    # packing: n must be a multiple of 128, output must not alias
    assert lib.exl3_pack(16, 128, 64, 3, 32, None) == L.EXL3_ERR_ARG
    assert lib.exl3_pack(16, 128, 128, 3, 16, None) == L.EXL3_ERR_ARG
    # router: too many experts, k > E
    assert lib.exl3_route(16, 2048, 1, 2048, 0, 8, None, None, None, 1.0, 1, 16, 0, 16, None, None) == \
        L.EXL3_ERR_UNSUPPORTED
    assert lib.exl3_route(16, 4, 1, 4, 0, 8, None, None, None, 1.0, 1, 16, 0, 16, None, None) == L.EXL3_ERR_ARG
    # MoE: missing workspace
    assert lib.exl3_moe_decode(16, 0, 128, 1, 16, 16, 2, 16, 4, 0, 128, 128, 0.0, 16, 2, None, 0, 0, None) == \
        L.EXL3_ERR_WORKSPACE
    assert lib.exl3_moe_gateup(1, 2, 16, 4, 0, 128, 128, 0.0, None, 0, 0, None) == L.EXL3_ERR_WORKSPACE
    # exl3_mgemm: k not a multiple of 128, A batches neither 1 nor the slot count, weighted slots not splitting
    # over the tokens, missing workspace

    def mgemm(k=128, a_batches=1, slots=2, weights=None, tokens=1, ws=None, ws_bytes=0):
        return lib.exl3_mgemm(16, 0, a_batches, k, 1, k, 128, 16, 16, 16, 16, 2, None, slots, weights, tokens, -1, -1,
                              16, 2, 128, ws, ws_bytes, None)
    assert mgemm(k=100) == L.EXL3_ERR_ARG
    assert mgemm(a_batches=3) == L.EXL3_ERR_ARG
    assert mgemm(weights=16, slots=3, tokens=2) == L.EXL3_ERR_ARG
    assert mgemm() == L.EXL3_ERR_WORKSPACE
    assert mgemm(slots=0) == L.EXL3_OK
    assert lib.exl3_mgemm_workspace_size(4, 8, 128, 128, 2) > lib.exl3_mgemm_workspace_size(2, 8, 128, 128, 2) > 0
    # negative group count
    assert gemv(groups=-1) == L.EXL3_ERR_ARG
    # zero rows is a no-op
    assert gemv(M=0) == L.EXL3_OK


def test_workspace_size_grows_with_batch():
    lib = L.lib()
    assert 0 < lib.exl3_gemv_workspace_size(1, 4096, 4096) < lib.exl3_gemv_workspace_size(8, 4096, 4096)
    a = lib.exl3_moe_workspace_size(1, 10, 512, 2048, 512, 0)
    b = lib.exl3_moe_workspace_size(4, 10, 512, 2048, 512, 1)
    assert 0 < a < b
    assert lib.exl3_moe_workspace_size(0, 10, 512, 2048, 512, 0) == 0


def test_ops_refuse_cpu_tensors():
    from exl3_b200 import ops
    x = torch.zeros(1, 128, dtype=torch.half)
    tr = torch.zeros(8, 8, 48, dtype=torch.int16)
    with pytest.raises(L.Exl3Error):
        ops.exl3_gemv(x, tr, torch.ones(128, dtype=torch.half), torch.ones(128, dtype=torch.half), 3,
                      torch.zeros(1, 128, dtype=torch.half))
    with pytest.raises(L.Exl3Error):
        ops.pack(tr, 3)
    with pytest.raises(L.Exl3Error):
        ops.route(torch.zeros(1, 16), 0, 2)


def test_bc_linear_rejects_unsupported_codebooks():
    from exl3_b200 import ops
    tr = torch.zeros(8, 8, 48, dtype=torch.int16)
    with pytest.raises(L.Exl3Error):
        ops.BC_LinearEXL3(tr, None, None, 3, None, True, False, None)
    with pytest.raises(L.Exl3Error):
        ops.BC_LinearEXL3(tr, None, None, 3.5, None, False, True, None)
    bc = ops.BC_LinearEXL3(tr, None, None, 3, None, False, True, None)
    assert (bc.in_features, bc.out_features) == (128, 128)
