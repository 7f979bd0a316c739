"""Failure detection on the GPU without a fault: a bounded in-kernel wait on a
barrier that nothing arrives on gives up, records its error word and returns;
the host reads the status and the context stays usable."""

from __future__ import annotations

import time
from pathlib import Path

import pytest
import torch

from strassen_tpu_b200 import _native


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_the_host_sees_it():
    import strassen_tpu_b200 as sb
    lib = _native.load()
    assert _native.device_status(reset=True) == 0
    start = time.perf_counter()
    _native.check(lib.sb_wait_selftest(torch.cuda.current_stream().cuda_stream))
    word = _native.device_status(reset=False)
    elapsed = time.perf_counter() - start
    header = (Path(__file__).resolve().parent.parent / "include" / "strassen_b200.h").read_text()
    assert "#define SB_SELFTEST_ERROR_CODE 9" in header
    assert word == 9
    assert 0.5 < elapsed < 30.0  # the wait's limit is 1 s of %globaltimer
    assert _native.device_status(reset=True) == 9
    assert _native.device_status() == 0
    # The context still runs work: an exact integer product.
    g = torch.Generator().manual_seed(4)
    a = torch.randint(-2, 3, (512, 512), generator=g).to(torch.bfloat16).cuda()
    b = torch.randint(-2, 3, (512, 512), generator=g).to(torch.bfloat16).cuda()
    got = sb.strassen_matmul(a, b, bm=256, bn=256, bk=256, output_dtype=torch.float32)
    assert torch.equal(got, a.float() @ b.float())
    assert _native.device_status() == 0
