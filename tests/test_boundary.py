"""The drop-in boundary, checked without a GPU.

* libkernel_lab_b200.so loads and exports every function ``include/kernel_lab_b200.h`` declares;
* calls that need no device (no-ops, argument validation) answer correctly;
* ``import kernel_lab._C`` registers kernel-lab's exact ``torch.ops.kernel_lab`` schemas
  (csrc/torch_bindings.cpp:107-113 there) and Meta kernels for tracing.
"""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest
import torch

from tests.conftest import REPO

HEADER = REPO / "include" / "kernel_lab_b200.h"
CUDA_ERROR_INVALID_VALUE = 1


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(kl_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_abi():
    names = declared_functions()
    assert names == [
        "kl_version",
        "kl_status_string",
        "kl_rms_norm",
        "kl_paged_decode_workspace_size",
        "kl_paged_decode",
        "kl_paged_decode_attention",
        "kl_paged_decode_read_status",
        "kl_paged_decode_gather",
        "kl_ipc_alloc",
        "kl_ipc_open",
        "kl_ipc_close",
        "kl_ipc_free",
        "kl_paged_decode_noalloc",
        "kl_paged_decode_noalloc_read_status",
        "kl_paged_kv_append",
        "kl_paged_decode_fp8",
        "kl_paged_kv_append_fp8",
        "kl_paged_decode_cascade_workspace_size",
        "kl_paged_decode_cascade",
    ]


def test_library_exports_every_declared_symbol():
    from kernel_lab import capi

    lib = capi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(capi.SIGNATURES) == set(declared_functions())
    nm = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r" T (kl_\w+)$", nm.stdout, flags=re.M))
    assert set(declared_functions()) <= exported


def test_version_and_status_strings():
    from kernel_lab import capi

    assert capi.version().startswith("kernel_lab_b200 ") and "sm_100a" in capi.version()
    assert capi.status_string(0) == "success"
    assert "invalid" in capi.status_string(CUDA_ERROR_INVALID_VALUE).lower()


def test_noop_and_validation_without_a_device():
    from kernel_lab import capi

    lib = capi.load()
    # rows == 0 and batch == 0 are no-ops (kernel-lab rmsnorm.cu:102, paged_attention.cu:187).
    assert lib.kl_rms_norm(2, None, None, None, None, 0, 4096, 4096, 1e-5, None) == 0
    assert lib.kl_paged_decode(2, *([None] * 6), 0, 32, 8, 128, 16, 4, 4, 10, 0.1, 0, None, 0, None, 0, None) == 0
    # Bad arguments are rejected before anything touches a device.
    assert lib.kl_rms_norm(2, None, None, None, None, 4, 4096, 4096, 1e-5, None) == CUDA_ERROR_INVALID_VALUE
    assert lib.kl_rms_norm(7, 1, 1, None, 1, 4, 4096, 4096, 1e-5, None) == CUDA_ERROR_INVALID_VALUE
    assert lib.kl_paged_decode(2, *([None] * 6), 4, 32, 8, 128, 16, 4, 4, 10, 0.1, 0, None, 0, None, 0, None) == (
        CUDA_ERROR_INVALID_VALUE
    )
    size = ctypes.c_size_t(1)
    assert lib.kl_paged_decode_workspace_size(2, 0, 32, 8, 128, 16, 4, 0, ctypes.byref(size), ctypes.byref(size)) == 0
    assert lib.kl_paged_decode_read_status(None, None, 0, None) == CUDA_ERROR_INVALID_VALUE
    # Append: batch 0 is a no-op; missing buffers or a row stride shorter than a row are rejected.
    assert lib.kl_paged_kv_append(2, *([None] * 6), 0, 8, 128, 16, 4, 4, 10, 1024, None, None) == 0
    assert lib.kl_paged_kv_append(2, *([None] * 6), 4, 8, 128, 16, 4, 4, 10, 1024, None, None) == (
        CUDA_ERROR_INVALID_VALUE
    )
    assert lib.kl_paged_kv_append(2, *([1] * 6), 4, 8, 128, 16, 4, 4, 10, 1000, None, None) == (
        CUDA_ERROR_INVALID_VALUE
    )
    # Cascade: batch 0 is a no-op; missing prefix tables, forced shapes off the tensor-core path
    # (fp32) and a prefix table narrower than its width are rejected before any launch.
    cas = lambda dt, batch, groups, ptr, d=128, pstride=4: lib.kl_paged_decode_cascade(  # noqa: E731
        dt, *([1] * 4), None, None, ptr, ptr, ptr, groups, pstride, 4, *([1] * 2), batch, 32, 8, d, 16, 4, 4, 10,
        0.1, 1, 1 << 20, 1, 1 << 20, None)
    assert cas(2, 0, 1, 1) == 0
    assert cas(2, 4, 1, None) == CUDA_ERROR_INVALID_VALUE
    assert cas(0, 4, 1, 1) == CUDA_ERROR_INVALID_VALUE
    assert cas(2, 4, 2, 1, pstride=3) == CUDA_ERROR_INVALID_VALUE
    assert lib.kl_paged_decode_cascade_workspace_size(2, 0, 1, 32, 8, 128, 16, 4, 4, ctypes.byref(size),
                                                      ctypes.byref(size)) == 0
    # Fused head gather: a rank outside the group, a missing peer output or flags, or a first epoch
    # of 0 is rejected before any launch; batch 0 with a valid descriptor is a no-op.
    g = capi.HeadGather()
    g.num_ranks, g.rank, g.epoch, g.done = 2, 0, 1, 1
    g.out[0], g.out[1], g.flags[0], g.flags[1] = 1, 1, 1, 1
    gat = lambda desc, batch: lib.kl_paged_decode_gather(  # noqa: E731
        2, ctypes.byref(desc), *([1] * 5), batch, 16, 4, 128, 16, 4, 4, 10, 0.1, 1, 1 << 20, 1, 1 << 20, None)
    assert gat(g, 0) == 0
    g.rank = 2
    assert gat(g, 4) == CUDA_ERROR_INVALID_VALUE
    g.rank, g.flags[1] = 0, None
    assert gat(g, 4) == CUDA_ERROR_INVALID_VALUE
    g.flags[1], g.epoch = 1, 0
    assert gat(g, 4) == CUDA_ERROR_INVALID_VALUE
    assert lib.kl_paged_decode_gather(2, None, *([1] * 5), 4, 16, 4, 128, 16, 4, 4, 10, 0.1, 1, 1, 1, 1, None) == (
        CUDA_ERROR_INVALID_VALUE
    )
    assert lib.kl_ipc_open(None, None) == CUDA_ERROR_INVALID_VALUE
    assert lib.kl_ipc_close(None) == 0 and lib.kl_ipc_free(None) == 0


# kernel-lab's schema strings, verbatim (csrc/torch_bindings.cpp:108-113 there).
REFERENCE_SCHEMAS = {
    "rms_norm": "rms_norm(Tensor! out, Tensor x, Tensor weight, float eps) -> ()",
    "fused_add_rms_norm": "fused_add_rms_norm(Tensor! out, Tensor x, Tensor! residual, Tensor weight, float eps) -> ()",
    "paged_decode_attention": (
        "paged_decode_attention(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, "
        "Tensor block_table, Tensor seq_lens, float scale) -> ()"
    ),
}


def test_torch_ops_have_the_reference_schemas():
    from kernel_lab import _C, cuda_ops  # noqa: F401

    for name, schema in REFERENCE_SCHEMAS.items():
        op = getattr(torch.ops.kernel_lab, name)
        assert str(op.default._schema) == str(torch._C.parse_schema("kernel_lab::" + schema))
    assert "num_splits" in str(torch.ops.kernel_lab.paged_decode_attention_splits.default._schema)
    for name in ("paged_decode_attention_fp8", "paged_kv_append_fp8", "paged_decode_attention_cascade"):
        assert "k_scale" in str(getattr(torch.ops.kernel_lab, name).default._schema)
    assert "prefix_indptr" in str(torch.ops.kernel_lab.paged_decode_attention_cascade.default._schema)
    assert str(torch.ops.kernel_lab.paged_kv_append.default._schema) == str(torch._C.parse_schema(
        "kernel_lab::paged_kv_append(Tensor! k_cache, Tensor! v_cache, Tensor k_new, Tensor v_new, "
        "Tensor block_table, Tensor positions) -> ()"))
    assert cuda_ops._LOADED


def test_meta_kernels_trace_without_a_device():
    from kernel_lab import _C  # noqa: F401

    x = torch.empty(4, 256, device="meta", dtype=torch.float16)
    w = torch.empty(256, device="meta", dtype=torch.float16)
    out = torch.empty_like(x)
    torch.ops.kernel_lab.rms_norm(out, x, w, 1e-6)
    torch.ops.kernel_lab.fused_add_rms_norm(out, x, torch.empty_like(x), w, 1e-6)
    q = torch.empty(2, 8, 64, device="meta", dtype=torch.bfloat16)
    kc = torch.empty(4, 16, 2, 64, device="meta", dtype=torch.bfloat16)
    bt = torch.empty(2, 2, device="meta", dtype=torch.int32)
    ln = torch.empty(2, device="meta", dtype=torch.int32)
    torch.ops.kernel_lab.paged_decode_attention(torch.empty_like(q), q, kc, kc, bt, ln, 0.125)
    kn = torch.empty(2, 2, 64, device="meta", dtype=torch.bfloat16)
    torch.ops.kernel_lab.paged_kv_append(kc, torch.empty_like(kc), kn, kn, bt, ln)
    pi = torch.empty(2, device="meta", dtype=torch.int32)
    torch.ops.kernel_lab.paged_decode_attention_cascade(torch.empty_like(q), q, kc, kc, bt, ln, pi[:1].expand(1),
                                                        bt, ln, 0.125)


def test_cuda_ops_fail_loudly_without_a_device():
    from kernel_lab import cuda_ops

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert not cuda_ops.available()
    with pytest.raises(RuntimeError):
        cuda_ops.rms_norm(torch.randn(2, 8), torch.ones(8))


def test_extensions_share_the_process_libstdcxx():
    """Neither shared object may carry its own copy of libstdc++: a second copy of the
    iostream/locale state crashes the first TORCH_CHECK that formats a number."""
    from kernel_lab import capi

    ext = next(capi.LIB_PATH.parent.glob("_C*.so"))
    for so in (capi.LIB_PATH, ext):
        nm = subprocess.run(["nm", "-C", "--defined-only", str(so)], capture_output=True, text=True, check=True)
        bad = re.findall(r" [TW] (std::(?:codecvt|basic_ostream|locale)\S*)", nm.stdout)
        assert not bad, f"{so.name} defines libstdc++ internals: {bad[:3]}"


def test_head_gather_descriptor_layout_matches_the_header(tmp_path):
    """capi.HeadGather mirrors kl_head_gather_t: the size and every field's offset, as a C compiler
    lays the header's struct out (gcc on the header itself), so a caller's descriptor is read
    field for field by the library."""
    import shutil

    from kernel_lab import capi

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    fields = ["num_ranks", "rank", "epoch", "out", "flags", "done", "timeout_ms"]
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "kernel_lab_b200.h"\nint main(void) {\n'
        '  printf("%zu", sizeof(kl_head_gather_t));\n'
        + "".join(f'  printf(" %zu", offsetof(kl_head_gather_t, {f}));\n' for f in fields)
        + "  return 0;\n}\n"
    )
    exe = tmp_path / "layout"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["gcc", f"-I{REPO / 'include'}", f"-I{cuda_inc}", str(src), "-o", str(exe)], check=True)
    c_size, *c_offsets = map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split())
    assert ctypes.sizeof(capi.HeadGather) == c_size
    assert [getattr(capi.HeadGather, f).offset for f in fields] == c_offsets


def test_build_reads_decode_spills_from_the_ptxas_report():
    """The build keeps the decode kernels' spill-free compilation by reading ptxas's -v report."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("kl_build", REPO / "kernel-lab_b200" / "build.py")
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    log = (
        "ptxas info    : Compiling entry function '_ZN3klb16decode_tc_kernelI13__nv_bfloat16Li128ELi1E' for 'sm_100a'\n"
        "ptxas info    : Function properties for _ZN3klb16decode_tc_kernelI13__nv_bfloat16Li128ELi1E\n"
        "    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads\n"
        "ptxas info    : Compiling entry function '_ZN3klb16decode_tc_kernelI6__halfLi128ELi2E' for 'sm_100a'\n"
        "    232 bytes stack frame, 852 bytes spill stores, 1364 bytes spill loads\n"
        "ptxas info    : Compiling entry function '_ZN3klb21rmsnorm_row_regs' for 'sm_100a'\n"
        "    0 bytes stack frame, 8 bytes spill stores, 8 bytes spill loads\n"
    )
    assert build.decode_spills(log) == {
        "_ZN3klb16decode_tc_kernelI13__nv_bfloat16Li128ELi1E": 0,
        "_ZN3klb16decode_tc_kernelI6__halfLi128ELi2E": 1364,
    }
