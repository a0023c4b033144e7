"""Failure detection on the GPU without faulting it.

The diagnostic flag NVFP4_FLAG_DIAG_SKIP_MMA makes the MMA issuer issue nothing, so no
stage is ever released and no accumulator is ever completed: the kernel's bounded
waits (about 2 s) run out, the CTAs record the reason in the workspace error word,
drain their in-flight copies, free TMEM and exit. The host reads the status through
nvfp4_workspace_check, and the same process must then run a normal launch correctly.
Nothing here traps, faults or hangs the device.
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu


def _table(pkg, prob):
    N = pkg._native
    t = np.zeros(prob.num_groups, dtype=N.GROUP_DTYPE)
    for key, lst in (("a", prob.a), ("b", prob.b), ("sfa", prob.sfa), ("sfb", prob.sfb),
                     ("c", prob.c)):
        t[key] = [x.data_ptr() for x in lst]
    t["m"] = prob.m
    t["n"] = prob.n
    t["k"] = prob.k
    t["alpha"] = 1.0
    t["alpha2"] = 1.0
    return t


@pytest.mark.parametrize("cta_flag", ["single", "pair"])
def test_stalled_pipeline_reports_timeout_and_context_survives(pkg, cta_flag):
    N = pkg._native
    prob = pkg.workloads.make_problem("stall", [256, 100], 256, 1024, seed=8, device="cuda")
    table = _table(pkg, prob)
    flags = N.FLAG_CTA_PAIR if cta_flag == "pair" else N.FLAG_SINGLE_CTA
    ws = torch.zeros(N.workspace_size(prob.num_groups), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    N.grouped_gemm_raw(table, flags | N.FLAG_DIAG_SKIP_MMA, ws.data_ptr(), ws.numel(), stream)
    with pytest.raises(N.Nvfp4Error) as err:
        N.workspace_check(ws.data_ptr(), stream)
    elapsed = time.time() - t0
    assert err.value.status == N.ERR_DEVICE_TIMEOUT
    assert "device error bits" in err.value.detail
    assert 1.0 < elapsed < 60.0, elapsed
    # The error word was cleared by the check, and the context is still usable.
    assert N.workspace_check(ws.data_ptr(), stream) == 0
    N.grouped_gemm_raw(table, flags, ws.data_ptr(), ws.numel(), stream)
    assert N.workspace_check(ws.data_ptr(), stream) == 0
    for g in range(prob.num_groups):
        exp = O.ref_gemm(prob.a[g].cpu().numpy(), prob.b[g].cpu().numpy(),
                         prob.sfa_plain[g].cpu().numpy(), prob.sfb_plain[g].cpu().numpy())
        assert O.compare_fp16(prob.c[g].cpu().numpy(), exp, None)["ok"]
