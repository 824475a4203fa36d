"""lx_flow_op_attention_static, the attention entry point that allocates no
device memory, through the C ABI.

It exists for callers that may not allocate on the call path (a
deadline-bound audio loop, an embedder that owns all of HBM through its own
pool): its scratch is fixed static device storage of the library.  Checked
here: two calls in a row on different shapes against the allocating entry
point lx_flow_op_attention (the second, smaller call must not see anything
the first left in the shared storage); the largest allowed call against a
float64 attention reference; that a call after the first leaves the device's
free memory unchanged; and that oversized calls are rejected.  This file is
collected last and passes alone in a fresh process as well as after the other
GPU tests."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import attn_ref_fp64, packed_starts, rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-6      # same kernels on the same inputs: expected bit-identical
FP64_TOL = 4e-3  # attention vs float64, bf16 output store (as in test_gpu_ops)


@pytest.fixture(scope="module")
def lib():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from larynx_b200 import flow
    flow.load_library()
    return flow


def _inputs(lengths, seed):
    R = packed_starts(lengths)[1]
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(R, 1024, generator=g) * 1.5).to(torch.bfloat16)
    k = (torch.randn(R, 1024, generator=g) * 1.5).to(torch.bfloat16)
    v = torch.randn(R, 1024, generator=g).to(torch.bfloat16)
    return R, q, k, v


def _valid_rows(lengths):
    starts, _ = packed_starts(lengths)
    return np.concatenate([np.arange(s, s + L) for s, L in zip(starts, lengths)])


def _pair(lib, lengths, chunk, seed):
    R, q, k, v = _inputs(lengths, seed)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    ref = torch.zeros(R, 1024, dtype=torch.bfloat16, device="cuda")
    got = torch.full((R, 1024), float("nan"), dtype=torch.bfloat16, device="cuda")
    lib.op_attention(lengths, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), ref.data_ptr(), chunk)
    lib.op_attention_static(lengths, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), got.data_ptr(), chunk)
    torch.cuda.synchronize()
    rows = _valid_rows(lengths)
    a, b = got.float().cpu().numpy()[rows], ref.float().cpu().numpy()[rows]
    assert np.isfinite(a).all()
    return rel_l2(a, b), (q, k, v, a)


def test_static_matches_allocating_entry_point_twice(lib):
    # largest allowed packed size first (4096 rows), then a smaller block-causal case
    L1 = [1000, 2000, 1096]
    e1, (q, k, v, got1) = _pair(lib, L1, 0, seed=11)
    e2, _ = _pair(lib, [300, 57, 129], 50, seed=12)
    assert e1 < TOL, e1
    assert e2 < TOL, e2
    # the 4096-row call (a 2000-frame sequence among them) against float64
    starts, _ = packed_starts(L1)
    ref = attn_ref_fp64(q.double().numpy(), k.double().numpy(), v.double().numpy(), L1, starts, 0)
    err = rel_l2(got1, ref[_valid_rows(L1)])
    assert err < FP64_TOL, err


def test_static_call_leaves_free_memory_unchanged(lib):
    """A call after the first (which may load the module and its static
    storage) must not grow any device allocation: free memory before and after
    is the same.  Inputs and outputs are allocated before the first reading."""
    lengths = [700, 1200]
    R, q, k, v = _inputs(lengths, seed=13)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    out = torch.empty(R, 1024, dtype=torch.bfloat16, device="cuda")
    lib.op_attention_static(lengths, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), 0)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    lib.op_attention_static(lengths, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), 0)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, (free0, free1)


def test_static_rejects_oversized_calls(lib):
    from larynx_b200.flow import FlowError
    p = 1 << 20   # never dereferenced: the size check fails before any device work
    with pytest.raises(FlowError, match="LX_ERR_ARG"):
        lib.op_attention_static([4097], p, p, p, p)          # 4104 packed rows
    with pytest.raises(FlowError, match="LX_ERR_ARG"):
        lib.op_attention_static([8] * 513, p, p, p, p)       # 513 sequences, 4104 rows
