"""Failure detection without a GPU fault: a device-side wait that can never
complete gives up after its bound, the kernel returns, the host reads
MP_ETIMEOUT through mp_sync_check, and the context keeps working (the
reference reports errors through `err` strings and empty buffers,
src/ming-dit.h:185-189; this build's equivalent is the status code)."""
import time

import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P
from mingproj._lib import MP_ETIMEOUT, MPError

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_recovers(ctx):
    t0 = time.perf_counter()
    ctx.selftest_wait(5_000_000)  # 5 ms: an mbarrier nobody arrives on
    with pytest.raises(MPError) as e:
        ctx.sync_check()
    elapsed = time.perf_counter() - t0
    assert e.value.status == MP_ETIMEOUT
    assert elapsed < 5.0, "the wait must end by its bound, not hang"
    ctx.sync_check()  # the error was reported once and cleared

    # the same context still runs a projection correctly
    rng = np.random.default_rng(77)
    m, n, k = 200, 256, 256
    pw = P.synthetic_affine(rng, n, k, 8)
    w = ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases)
    x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    y = ctx.linear(w, xd)
    ctx.sync_check()
    ref = O.projection(x, pw.data, pw.scales, pw.biases, n, k, 8, False)
    err = O.rel_l2(y.float().cpu().numpy().astype(np.float64), ref)
    w.free()
    assert err <= 5e-3
