"""The no-allocation entry point ``sb_strassen_gemm_norm_residual_noalloc``.

It serves callers that cannot give this library scratch memory or let it call
cudaMalloc -- e.g. a custom-call handler inside a framework that owns the
device memory, or a service with a fixed memory budget -- by keeping the fp32
pre-norm rows of the norm_residual_add epilogue in a 32 MiB device array
built into the library.  The test calls it through the C ABI twice in a row
(the array keeps the previous call's contents between calls) and compares each
result with the ordinary entry point, which uses a caller workspace.  It also
checks that a problem larger than the array is refused before any launch.
This file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import strassen_ref as ref

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

MAX_ABS_REL_RMS = 2e-2  # the parity bar used by the other GPU tests


def _dev(x):
    bits = ref.bf16_bits(np.asarray(x, np.float32)).view(np.int16)
    return torch.from_numpy(bits.copy()).view(torch.bfloat16).cuda()


def _epilogue(residual, scale, eps=1e-6):
    from strassen_tpu_b200._native import SB_BF16, SbEpilogue
    ep = SbEpilogue()
    ep.kind = 6  # SB_EPI_NORM_RESIDUAL_ADD
    ep.residual = residual.data_ptr()
    ep.ld_residual = residual.stride(0)
    ep.residual_dtype = SB_BF16
    ep.aux_dtype = SB_BF16
    ep.norm_scale = scale.data_ptr()
    ep.norm_eps = eps
    return ep


def _noalloc(a, b, residual, scale, bm=256, bk=256):
    from strassen_tpu_b200 import _native
    m, k = a.shape
    n = b.shape[1]
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    ep = _epilogue(residual, scale)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = _native.load().sb_strassen_gemm_norm_residual_noalloc(
        stream, a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, a.stride(0), b.stride(0),
        out.stride(0), bm, n, bk, ctypes.byref(ep))
    _native.check(status)
    return out


def test_noalloc_matches_workspace_entry_point_twice_in_a_row():
    import strassen_tpu_b200 as sb
    m, k, n = 512, 768, 1024
    b = _dev(ref.normal_bf16((k, n), 902))
    scale = _dev(ref.bf16_round(1.0 + 0.02 * ref.normal_bf16((n,), 903)))
    for call, seed in enumerate((904, 905)):
        a = _dev(ref.normal_bf16((m, k), seed))
        residual = _dev(ref.normal_bf16((m, n), seed + 10))
        got = _noalloc(a, b, residual, scale)
        want = sb.strassen_matmul(a, b, bm=256, bn=n, bk=256, epilogue="norm_residual_add",
                                  residual=residual, norm_scale=scale)
        torch.cuda.synchronize()
        g = got.float().cpu().numpy().astype(np.float64)
        w = want.float().cpu().numpy().astype(np.float64)
        rms = np.sqrt(np.mean(w ** 2))
        assert np.isfinite(g).all(), f"call {call}"
        assert np.abs(g - w).max() <= MAX_ABS_REL_RMS * rms, f"call {call}"
    from strassen_tpu_b200 import _native
    assert _native.device_status() == 0


def test_noalloc_refuses_problems_beyond_its_scratch():
    from strassen_tpu_b200 import _native
    m, k, n = 4096, 256, 4096  # 16M fp32 values > 8M capacity
    a = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(k, n, dtype=torch.bfloat16, device="cuda")
    residual = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    scale = torch.ones(n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.StrassenError, match="exceeds the no-allocation scratch capacity"):
        _noalloc(a, b, residual, scale)


def test_noalloc_at_exact_capacity_and_one_row_tile_over():
    """M*N equal to the array's 8,388,608 fp32 values uses its last rows and is
    accepted (matching the workspace entry point); one more 256-row tile is
    refused before any launch."""
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    m, k, n = 2048, 256, 4096  # m * n == 8,388,608
    a = _dev(ref.normal_bf16((m, k), 906))
    b = _dev(ref.normal_bf16((k, n), 907))
    residual = _dev(ref.normal_bf16((m, n), 908))
    scale = _dev(ref.bf16_round(1.0 + 0.02 * ref.normal_bf16((n,), 909)))
    got = _noalloc(a, b, residual, scale)
    want = sb.strassen_matmul(a, b, bm=256, bn=n, bk=256, epilogue="norm_residual_add",
                              residual=residual, norm_scale=scale)
    torch.cuda.synchronize()
    g = got.float().cpu().numpy().astype(np.float64)
    w = want.float().cpu().numpy().astype(np.float64)
    rms = np.sqrt(np.mean(w ** 2))
    assert np.isfinite(g).all()
    assert np.abs(g - w).max() <= MAX_ABS_REL_RMS * rms
    assert _native.device_status() == 0
    m_over = m + 256
    a2 = torch.zeros(m_over, k, dtype=torch.bfloat16, device="cuda")
    r2 = torch.zeros(m_over, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.StrassenError, match="exceeds the no-allocation scratch capacity"):
        _noalloc(a2, b, r2, scale)
