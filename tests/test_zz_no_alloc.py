"""lx_flow_op_attention_static (the attention entry point that allocates no
device memory) against lx_flow_op_attention on the same inputs, through the
C ABI.  Two calls in a row on different shapes: the second, smaller call must
not see anything the first left in the shared static storage.  Runs alone in
a fresh process as well as after the other GPU tests."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-6   # same kernels on the same inputs: expected bit-identical


@pytest.fixture(scope="module")
def lib():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from larynx_b200 import flow
    flow.load_library()
    return flow


def _inputs(lengths, seed):
    R = sum((L + 7) // 8 * 8 for L in lengths)
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(R, 1024, generator=g) * 1.5).to(torch.bfloat16).cuda()
    k = (torch.randn(R, 1024, generator=g) * 1.5).to(torch.bfloat16).cuda()
    v = torch.randn(R, 1024, generator=g).to(torch.bfloat16).cuda()
    return R, q, k, v


def _pair(lib, lengths, chunk, seed):
    R, q, k, v = _inputs(lengths, seed)
    ref = torch.zeros(R, 1024, dtype=torch.bfloat16, device="cuda")
    got = torch.full((R, 1024), float("nan"), dtype=torch.bfloat16, device="cuda")
    lib.op_attention(lengths, q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), chunk)
    lib.op_attention_static(lengths, q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), chunk)
    torch.cuda.synchronize()
    starts = np.cumsum([0] + [(L + 7) // 8 * 8 for L in lengths])[:-1]
    rows = np.concatenate([np.arange(s, s + L) for s, L in zip(starts, lengths)])
    a, b = got.float().cpu().numpy()[rows], ref.float().cpu().numpy()[rows]
    assert np.isfinite(a).all()
    return rel_l2(a, b)


def test_static_matches_allocating_entry_point_twice(lib):
    # largest allowed packed size first, then a smaller block-causal case
    e1 = _pair(lib, [1000, 2000, 1096], 0, seed=11)
    e2 = _pair(lib, [300, 57, 129], 50, seed=12)
    assert e1 < TOL, e1
    assert e2 < TOL, e2


def test_static_rejects_oversized_calls(lib):
    from larynx_b200.flow import FlowError
    p = 1 << 20   # never dereferenced: the size check fails before any device work
    with pytest.raises(FlowError, match="LX_ERR_ARG"):
        lib.op_attention_static([4097], p, p, p, p)          # 4104 packed rows
    with pytest.raises(FlowError, match="LX_ERR_ARG"):
        lib.op_attention_static([8] * 513, p, p, p, p)       # 513 sequences, 4104 rows
