"""The tensor-core kernel's failure path on the GPU, without a GPU fault.

Every pipeline wait of the decode kernel is bounded. Through the test hook
(``qsa_b200_testing_set_wait_limit_ns``) the limit is cut to 1 ns, so that the
first wait that has to spin gives up: the CTA records code 1 in the device
error word, raises its abort flag so the other roles leave their loops, waits
(with the normal 1 s limit) for its own copies and MMAs in flight, frees its
tensor memory and returns. The host reads the word; the context stays usable
and the next call with the normal limit is correct again.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import bits, check_close, oracle_subset

pytestmark = pytest.mark.gpu

# (workload config, overrides, rows): unsplit rows (the static item walk),
# split rows whose chunks go out as partials to the combine kernel (fewer than
# two (row, KV head) pairs per SM: 32 rows x 8 KV heads), and split rows
# merged inside the CTA (the claimed walk with its named-barrier votes)
SHAPES = {
    "unsplit": (1, {}, 64),
    "split_partials": (0, dict(ppr=100, topk=1500, mode="sample"), 32),
    "split_merged": (4, dict(ppr=160, topk=2048, len_lo=64, len_hi=2048), 320),
}


@pytest.fixture(autouse=True)
def _restore_limit():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qsa_b200 import capi

    capi.device_error(clear=True)
    yield
    capi.testing_set_wait_limit_ns(0)
    capi.device_error(clear=True)


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_wait_that_runs_out_is_reported_and_the_next_call_is_correct(name):
    from qsa_b200 import capi, ops, qsa_decode
    from qsa_b200.inputs import make_workload

    cfg, over, rows = SHAPES[name]
    w = make_workload(cfg, "cuda", seed=7, rows=rows, **over)
    merged = ops.tc_merges_chunks(w.rows, w.meta["hq"], w.meta["hkv"], w.meta["topk"],
                                  torch.cuda.get_device_properties(0).multi_processor_count)
    assert merged == (name == "split_merged")
    out = torch.zeros_like(w.q)

    assert capi.testing_set_wait_limit_ns(1) == 10**9
    qsa_decode(*w.args(), out=out, kernel="tc")
    torch.cuda.synchronize()  # the kernel returned: no hang, no fault
    assert capi.testing_set_wait_limit_ns(0) == 1
    assert capi.device_error() == 1
    with pytest.raises(RuntimeError, match="device-side failure"):
        capi.check_device_error(clear=True)
    assert capi.device_error() == 0

    # the same call with the normal limit, on the same context
    qsa_decode(*w.args(), out=out, kernel="tc")
    torch.cuda.synchronize()
    capi.check_device_error()
    sample = list(range(0, w.rows, max(1, w.rows // 8)))
    check_close(bits(out[sample]), oracle_subset(w, sample), what=f"{name} after the timeout")
