"""CPU: the native libraries load, export what include/qsa_b200.h declares,
and reject bad arguments before touching a device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from conftest import PKG_ROOT, REPO

HEADER = REPO / "include" / "qsa_b200.h"
HEADERS = sorted((REPO / "include").glob("*.h"))


def _declared_functions(headers=None):
    text = "\n".join(h.read_text() for h in (headers or HEADERS))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b([A-Za-z_]\w*)\s*\(", text, flags=re.M)
    return sorted({n for n in names if n not in ("if", "defined")})


def test_header_declares_the_abi():
    names = _declared_functions()
    assert "qsa_b200_decode" in names and "launch_qsa_cuda" in names and "qsa_b200_slots" in names


def test_library_exports_every_declared_symbol():
    from qsa_b200 import capi

    lib = capi.lib()
    declared = _declared_functions()
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(capi.EXPORTED) | set(capi.TESTING_EXPORTED)
    assert set(_declared_functions([HEADER])) == set(capi.EXPORTED)
    assert lib.qsa_b200_abi_version() == 1


def test_library_exports_only_the_c_abi():
    """Internal C++ helpers stay hidden: the .so's dynamic symbol table
    exports exactly the declared C functions (plus nothing named qsa::*)."""
    import subprocess

    so = PKG_ROOT / "qsa_b200" / "libqsa_b200.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True, check=True).stdout
    text_syms = {l.split()[-1] for l in out.splitlines() if l.split()[1:2] == ["T"]}
    ours = {s for s in text_syms if "qsa" in s or s == "launch_qsa_cuda"}
    assert ours == set(_declared_functions()), sorted(ours)


def test_status_strings():
    from qsa_b200 import capi

    assert capi.status_string(0) == "ok"
    for code in range(-8, 0):
        assert capi.status_string(code) != "unknown status"


def _args_cpu(**over):
    from qsa_b200 import capi

    a = capi.DecodeArgs()
    a.rows, a.num_q_heads, a.num_kv_heads, a.head_dim = 4, 32, 8, 128
    a.page_size, a.pages_per_req, a.num_reqs, a.num_pages = 16, 4, 4, 16
    a.topk, a.indices_stride, a.btable_stride = 64, 64, 4
    a.softmax_scale, a.k_scale, a.v_scale = 128 ** -0.5, 1.0, 1.0
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,code", [
    (dict(head_dim=64), -3),
    (dict(num_q_heads=30), -2),
    (dict(num_q_heads=8 * 33), -3),
    (dict(rows=-1), -2),
    (dict(topk=-1), -2),
    (dict(page_size=0), -2),
    (dict(indices_stride=10), -2),
    (dict(btable_stride=2), -2),
    (dict(kernel=7), -3),
    # tensor-core kernel limits: 2^24 pages x 16 x 8 KV heads = 2^31 rows of
    # 128 bytes; 2^24 rows x 8 KV heads x 8 chunks = 2^30 work items
    (dict(num_pages=1 << 24), -3),
    (dict(num_pages=1 << 24, kernel=1), -3),
    (dict(rows=1 << 24, num_reqs=1 << 24, topk=4096, indices_stride=4096), -3),
])
def test_validation_errors(over, code):
    from qsa_b200 import capi

    a = _args_cpu(**over)
    # pointers are set so that only the field under test is wrong
    a.indices = a.btable = a.q = a.k_cache = a.v_cache = a.gate = a.out = ctypes.c_void_p(4096)
    assert capi.workspace_bytes(a) == code
    assert capi.decode(a) == code


def test_null_and_misaligned_pointers_are_rejected():
    from qsa_b200 import capi

    a = _args_cpu()
    assert capi.decode(a) == capi.ERR_NULL_POINTER
    a.indices = a.btable = a.q = a.k_cache = a.v_cache = a.gate = a.out = ctypes.c_void_p(4096)
    a.q = ctypes.c_void_p(4096 + 8)
    assert capi.decode(a) == capi.ERR_MISALIGNED
    a.q = ctypes.c_void_p(4096)
    a.indices = ctypes.c_void_p(4096 + 2)
    assert capi.decode(a) == capi.ERR_MISALIGNED


def test_empty_batch_is_a_no_op_without_a_device():
    from qsa_b200 import capi

    a = _args_cpu(rows=0)
    assert capi.decode(a) == capi.OK


def test_workspace_sizes():
    """[row map, tile flags, claim counter (tensor-core kernel)][partial
    outputs][partial lse], each 256-byte aligned; the CUDA-core kernel needs
    no row map."""
    from qsa_b200 import capi, ops

    a = _args_cpu(topk=512, indices_stride=512)
    a.indices = a.btable = a.q = a.k_cache = a.v_cache = a.gate = a.out = ctypes.c_void_p(4096)
    rowmap = 4 * 512 * 4 + 256 + 256
    assert capi.workspace_bytes(a) == rowmap == ops.workspace_bytes(4, 32, 8, 512)
    a.kernel = capi.KERNEL_SIMT
    assert capi.workspace_bytes(a) == 0 == ops.workspace_bytes(4, 32, 8, 512, kernel="simt")
    a.kernel = capi.KERNEL_AUTO
    a.topk, a.indices_stride = 1100, 1101
    n = 4 * 32 * 3
    rowmap = 4 * 3 * 512 * 4 + 256 + 256
    assert capi.workspace_bytes(a) == rowmap + n * 512 + n * 4 == ops.workspace_bytes(4, 32, 8, 1100)
    a256 = lambda x: -(-x // 256) * 256
    for hq in (128, 96, 72, 256, 136):  # groups 16, 12, 9, 32, 17: tensor-core kernel, 512-entry chunks
        a.num_q_heads = hq
        n = 4 * hq * 3
        assert capi.workspace_bytes(a) == rowmap + n * 512 + a256(n * 4) == ops.workspace_bytes(4, hq, 8, 1100)
    a.num_q_heads, a.kernel = 136, capi.KERNEL_SIMT  # the CUDA-core kernel: no row map
    n = 4 * 136 * 3
    assert capi.workspace_bytes(a) == n * 512 + a256(n * 4) == ops.workspace_bytes(4, 136, 8, 1100, kernel="simt")
    a.kernel = capi.KERNEL_AUTO
    # enough (row, KV head) pairs for the decode kernel to merge the chunks
    # itself (at least two per SM): no partials
    a.num_q_heads, a.rows, a.num_reqs = 32, 1024, 1024
    a.num_pages = 1024 * a.pages_per_req
    rowmap = 1024 * 3 * 512 * 4 + a256(1024 * 3 * 16) + 256
    assert capi.workspace_bytes(a) == rowmap == ops.workspace_bytes(1024, 32, 8, 1100, sm_count=148)
    a.kernel = capi.KERNEL_SIMT  # the CUDA-core kernel always writes partials
    n = 1024 * 32 * 3
    assert capi.workspace_bytes(a) == n * 512 + a256(n * 4) == ops.workspace_bytes(1024, 32, 8, 1100,
                                                                                     kernel="simt")


def test_torch_ops_register_and_refuse_cpu_tensors():
    import qsa_b200

    ops = qsa_b200.load_torch_ops()
    assert hasattr(ops, "decode") and hasattr(ops, "slots")
    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 16, 8, 128, dtype=torch.uint8)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    idx = torch.zeros(1, 4, dtype=torch.int32)
    with pytest.raises((RuntimeError, NotImplementedError)):
        qsa_b200.qsa_decode(q, k, k, 1.0, 1.0, bt, None, idx, q)


def test_product_never_imports_the_oracle():
    """Nothing under the package imports, loads or reads oracle/ (the checker
    stays a checker)."""
    pat = re.compile(r"\b(from|import)\s+oracle\b|oracle/|oracle\.|_ref\b")
    files = list((PKG_ROOT / "qsa_b200").glob("*.py")) + list((PKG_ROOT / "csrc").glob("*"))
    assert files
    for path in files:
        assert not pat.search(path.read_text()), path


def test_merge_policy_mirror():
    """The Python mirror of the decode's rule for merging split rows in the
    CTA: configs[4] (1024 rows, G = 8, 4 chunks) merges; a 12-row shard, a
    group of 16, a single chunk or more than 32 chunks do not."""
    from qsa_b200 import ops

    assert ops.tc_merges_chunks(1024, 64, 8, 2048, 148)
    assert not ops.tc_merges_chunks(12, 64, 8, 2048, 148)
    assert not ops.tc_merges_chunks(1024, 128, 8, 2048, 148)
    assert not ops.tc_merges_chunks(1024, 64, 8, 512, 148)
    assert not ops.tc_merges_chunks(1024, 64, 8, 512 * 33, 148)
    assert ops.tc_merges_chunks(37, 32, 8, 1600, 148) and not ops.tc_merges_chunks(36, 32, 8, 1600, 148)


def test_group_support_mirror_matches_the_library():
    """ops.tc_supports_group (used to size workspaces on the Python side)
    agrees with the library for every group size: the tensor-core kernel
    takes 1 to 32 and refuses the others."""
    from qsa_b200 import capi, ops

    for g in range(1, 34):
        a = _args_cpu(num_q_heads=8 * g, kernel=capi.KERNEL_TC)
        a.indices = a.btable = a.q = a.k_cache = a.v_cache = a.gate = a.out = ctypes.c_void_p(4096)
        got = capi.workspace_bytes(a)
        assert (got >= 0) == ops.tc_supports_group(g), (g, got)
        if got < 0:
            assert got == capi.ERR_UNSUPPORTED
