"""Failure detection on the device, tested without a GPU fault.

Every wait in the library's kernels is bounded (2 s); when one runs out the
kernel records an error code, its roles leave through the CTA's abort flag,
the tensor memory is freed and the host call returns LX_ERR_TIMEOUT.  Here
lx_flow_selftest_wait makes such a wait run out on purpose (a producer that
never arrives, a limit of a few milliseconds), and the test checks the status,
the error code, and that the same process keeps computing correct results
afterwards."""

import time

import pytest

torch = pytest.importorskip("torch")

from conftest import rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu
LX_OK, LX_ERR_TIMEOUT = 0, 7


@pytest.fixture(scope="module")
def flow():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from larynx_b200 import flow
    flow.load_library()
    return flow


def test_wait_completes_when_the_producer_arrives(flow):
    assert flow.selftest_wait(True, 5.0) == (LX_OK, 0)


def test_wait_runs_out_and_the_context_recovers(flow):
    t0 = time.perf_counter()
    rc, code = flow.selftest_wait(False, 2.0)
    dt = time.perf_counter() - t0
    assert rc == LX_ERR_TIMEOUT
    assert code == 3            # the consumer gave up first; the second waiter left through the abort flag
    assert dt < 1.0, dt         # 2 ms limit plus 1 ms suspend steps, not the kernels' 2 s
    # the same context still computes: a GEMM through the C ABI, then the test again
    g = torch.Generator().manual_seed(5)
    A = torch.randn(256, 1024, generator=g).to(torch.bfloat16)
    B = (torch.randn(1024, 1024, generator=g) * 0.05).to(torch.bfloat16)
    Ad, Bd = A.cuda(), B.cuda()
    C = torch.empty(256, 1024, device="cuda")
    flow.op_gemm(256, 1024, 1024, Ad.data_ptr(), Bd.data_ptr(), 0, C.data_ptr())
    torch.cuda.synchronize()
    assert rel_l2(C.cpu().numpy(), (A.double() @ B.double().T).numpy()) < 1e-5
    assert flow.selftest_wait(True, 5.0) == (LX_OK, 0)
    assert flow.selftest_wait(False, 1.0)[0] == LX_ERR_TIMEOUT


def test_selftest_rejects_bad_limits(flow):
    assert flow.selftest_wait(False, 0.0)[0] == 1       # LX_ERR_ARG, nothing launched
    assert flow.selftest_wait(False, 5000.0)[0] == 1
