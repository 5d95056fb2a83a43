"""Fused residual-add + RMSNorm on the GPU vs the reference's golden vectors and the oracle.

The updated residual must match bit for bit (kernel-lab tests/test_rmsnorm.py:35 and
tests/test_cuda_kernels.py:33); the normalised output within kernel-lab's per-dtype
tolerance. Calls go through the C ABI and through the drop-in torch ops.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import (
    DT,
    DT_NAME,
    assert_within_abs_or_ulp,
    golden_array,
    golden_index,
    golden_to_torch,
    make_rms_inputs,
    sha,
    to_f32_numpy,
    tolerance,
)

pytestmark = pytest.mark.gpu

RMS_CASES = [c["name"] for c in golden_index()["rmsnorm"]]


def _case(name):
    return next(c for c in golden_index()["rmsnorm"] if c["name"] == name)


@pytest.mark.parametrize("name", RMS_CASES)
@pytest.mark.parametrize("path", ["capi", "op"])
def test_golden_cases(name, path):
    from kernel_lab import capi, cuda_ops

    case = _case(name)
    dt = case["dt"]
    x, r, w = (t.cuda() for t in make_rms_inputs(case["shape"], DT[dt]))
    if path == "capi":
        out = torch.empty_like(x)
        res = r.clone()
        capi.rms_norm(out, x, w, case["eps"], residual=res)
        plain = torch.empty_like(x)
        capi.rms_norm(plain, x, w, case["eps"])
    else:
        out, res = cuda_ops.fused_add_rms_norm(x, r, w, case["eps"])
        plain = cuda_ops.rms_norm(x, w, case["eps"])
    torch.cuda.synchronize()
    assert sha(res) == case["residual_out_sha256"]  # bit-exact residual
    h = case["shape"][-1]
    if "sample_rows" in case:
        rows = case["sample_rows"]
        want = golden_to_torch(golden_array("rmsnorm", f"{name}/out_rows"), dt).cuda()
        want_plain = golden_to_torch(golden_array("rmsnorm", f"{name}/out_plain_rows"), dt).cuda()
        torch.testing.assert_close(out.reshape(-1, h)[rows], want, **tolerance(DT[dt]))
        torch.testing.assert_close(plain.reshape(-1, h)[rows], want_plain, **tolerance(DT[dt]))
        # Every row against the unrounded fp32 oracle: north-star bound (bf16 2e-2), or one
        # bf16 ulp where that is larger (|y| >= 4: the two nearest bf16 values are 2^-5 apart).
        _, res32 = oracle.fused_add_rms_norm(to_f32_numpy(x), to_f32_numpy(r), to_f32_numpy(w), case["eps"], dt)
        exact = oracle.rms_norm(res32, to_f32_numpy(w), case["eps"], "f32")
        assert_within_abs_or_ulp(out, exact, torch.bfloat16)
    else:
        want = golden_to_torch(golden_array("rmsnorm", f"{name}/out"), dt).cuda()
        want_plain = golden_to_torch(golden_array("rmsnorm", f"{name}/out_plain"), dt).cuda()
        torch.testing.assert_close(out, want, **tolerance(DT[dt]))
        torch.testing.assert_close(plain, want_plain, **tolerance(DT[dt]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 64), (3, 100), (8, 4096), (2, 5, 8192), (3, 16384), (2, 40000), (5, 72)])
def test_shapes_against_oracle(shape, dtype):
    """kernel-lab's CUDA test shapes (tests/test_cuda_kernels.py:17-22) plus rows wider than
    the register path and odd widths."""
    from kernel_lab import cuda_ops

    x, r, w = (t.cuda() for t in make_rms_inputs(shape, dtype, seed=1))
    out, res = cuda_ops.fused_add_rms_norm(x, r, w, 1e-5)
    ref_out, ref_res = oracle.fused_add_rms_norm(to_f32_numpy(x), to_f32_numpy(r), to_f32_numpy(w), 1e-5, DT_NAME[dtype])
    np.testing.assert_array_equal(res.float().cpu().numpy(), ref_res)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref_out, **tolerance(dtype))
    plain = cuda_ops.rms_norm(x, w, 1e-5)
    np.testing.assert_allclose(
        plain.float().cpu().numpy(), oracle.rms_norm(to_f32_numpy(x), to_f32_numpy(w), 1e-5, DT_NAME[dtype]),
        **tolerance(dtype),
    )


def test_unaligned_rows_take_the_scalar_path():
    """kernel-lab tests/test_cuda_kernels.py:37-41: misaligned start and odd width."""
    from kernel_lab import cuda_ops

    base = torch.randn(4, 130, device="cuda", dtype=torch.float16)
    x = base[:, 1:101]
    w = torch.randn(100, device="cuda", dtype=torch.float16)
    want = oracle.rms_norm(to_f32_numpy(x), to_f32_numpy(w), 1e-6, "f16")
    np.testing.assert_allclose(cuda_ops.rms_norm(x, w).float().cpu().numpy(), want, **tolerance(torch.float16))


def test_strided_rows_are_supported():
    from kernel_lab import cuda_ops

    base = torch.randn(4, 192, device="cuda")
    x = base[:, :128]  # row stride 192
    w = torch.ones(128, device="cuda")
    want = oracle.rms_norm(to_f32_numpy(x), to_f32_numpy(w), 1e-6, "f32")
    np.testing.assert_allclose(cuda_ops.rms_norm(x, w).cpu().numpy(), want, atol=1e-5, rtol=1e-5)


def test_inputs_are_not_modified_and_zero_rows_stay_finite():
    from kernel_lab import cuda_ops

    x, r, w = (t.cuda() for t in make_rms_inputs((3, 64), torch.float32))
    x0, r0 = x.clone(), r.clone()
    cuda_ops.fused_add_rms_norm(x, r, w)
    assert torch.equal(x, x0) and torch.equal(r, r0)
    z = torch.zeros(2, 4096, device="cuda", dtype=torch.bfloat16)
    assert torch.isfinite(cuda_ops.rms_norm(z, torch.ones(4096, device="cuda", dtype=torch.bfloat16))).all()


def test_in_place_op_updates_residual():
    from kernel_lab import cuda_ops  # noqa: F401

    x, r, w = (t.cuda() for t in make_rms_inputs((16, 8192), torch.bfloat16))
    want_out, want_res = oracle.fused_add_rms_norm(to_f32_numpy(x), to_f32_numpy(r), to_f32_numpy(w), 1e-5, "bf16")
    out = torch.empty_like(x)
    torch.ops.kernel_lab.fused_add_rms_norm(out, x, r, w, 1e-5)
    np.testing.assert_array_equal(r.float().cpu().numpy(), want_res)
    np.testing.assert_allclose(out.float().cpu().numpy(), want_out, **tolerance(torch.bfloat16))


def test_validation_errors():
    from kernel_lab import cuda_ops

    x = torch.randn(2, 32, device="cuda")
    with pytest.raises(RuntimeError, match="weight size"):
        cuda_ops.rms_norm(x, torch.ones(16, device="cuda"))
    with pytest.raises(RuntimeError, match="residual"):
        cuda_ops.fused_add_rms_norm(x, torch.randn(2, 16, device="cuda"), torch.ones(32, device="cuda"))
