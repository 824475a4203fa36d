"""The pre-laid-out weight cache: a model loaded from a layout file written by
lx_flow_save_layout decodes bit-identically to the model loaded from the
flow.gguf it came from; malformed files are rejected."""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    from larynx_b200.weights import write_synthetic_gguf
    p = str(tmp_path_factory.mktemp("w") / "flow_synth.gguf")
    write_synthetic_gguf(p, seed=0, std=0.02)
    return p


def _decode(dec, seed=5):
    rng = np.random.default_rng(seed)
    L = np.array([150, 77, 301], np.int32)
    n = int(L.sum())
    mu, cond, noise = (rng.standard_normal(80 * n).astype(np.float32) for _ in range(3))
    spks = rng.standard_normal((len(L), 80)).astype(np.float32)
    return dec.decode(L, mu, cond, spks, noise=noise)


def test_layout_roundtrip_is_bit_identical(gguf_path, tmp_path):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    from larynx_b200 import FlowDecoder
    a = FlowDecoder(0)
    t0 = time.perf_counter()
    assert a.load(gguf_path), a.last_error
    t_gguf = time.perf_counter() - t0
    lay = str(tmp_path / "flow.lxfl")
    assert a.save_layout(lay), a.last_error
    b = FlowDecoder(0)
    t0 = time.perf_counter()
    assert b.load_layout(lay), b.last_error
    t_layout = time.perf_counter() - t0
    ra, rb = _decode(a), _decode(b)
    np.testing.assert_array_equal(ra, rb)
    # the estimator at an arbitrary t uses the fp32 AdaLN weights of the file
    print(f"load: gguf {t_gguf:.2f} s, layout {t_layout:.2f} s")
    a.close()
    b.close()


def test_layout_rejects_bad_files(tmp_path):
    from larynx_b200 import FlowDecoder
    d = FlowDecoder(0)
    assert not d.load_layout(str(tmp_path / "missing.lxfl"))
    bad = tmp_path / "bad.lxfl"
    bad.write_bytes(b"LXFL" + b"\x02\x00\x00\x00" + b"\x00" * 200)  # wrong version
    assert not d.load_layout(str(bad))
    assert "layout" in d.last_error
    d.close()
