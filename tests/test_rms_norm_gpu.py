"""rms_norm on the GPU through the C ABI, the torch binding and the plugins, against
the oracle (a restatement of the zoo golden) and the reference's python golden
samples.  Bar: residual_out bit-exact; output within one step of the 16-bit type
of the oracle (the kernel's sum of squares runs in another order)."""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp(v, dtype):
    mant = 10 if dtype == "f16" else 7
    a = np.maximum(np.abs(v.astype(np.float32)), np.float32(2.0 ** -14))
    return np.exp2(np.floor(np.log2(a)) - mant)


def _run_capi(c, x, w, r):
    from gpu_util import handle, words_to_dev
    from tecoops import capi
    dx, dw = words_to_dev(x, c["dtype"]), words_to_dev(w, c["dtype"])
    dr = words_to_dev(r, c["dtype"]) if r is not None else None
    out = torch.empty_like(dx)
    ro = torch.empty_like(dx) if r is not None else None
    dt = None if c["dtype"] == "f16" else capi.DATA_BFLOAT16
    capi.check(capi.rms_norm(handle(), dx.data_ptr(), dw.data_ptr(),
                             dr.data_ptr() if dr is not None else 0, out.data_ptr(),
                             ro.data_ptr() if ro is not None else 0, c["N"], c["D"], c["eps"],
                             dtype=dt), "tecoopsRmsNorm")
    torch.cuda.synchronize()
    return out, ro


@pytest.mark.parametrize("name", sorted(cases.RMS_CASES))
def test_rms_norm_vs_oracle_and_golden(golden, name):
    from gpu_util import dev_to_words
    c = cases.RMS_CASES[name]
    x, w, r = cases.rms_inputs(c)
    out, ro = _run_capi(c, x, w, r)
    ey, ero = oracle.rms_norm(x, w, r, c["eps"], c["dtype"])
    yo = seeded.words_to_f32(dev_to_words(out), c["dtype"])
    ye = seeded.words_to_f32(ey, c["dtype"])
    assert np.isfinite(yo).all()
    assert np.all(np.abs(yo - ye) <= _ulp(ye, c["dtype"]) + 1e-7), np.abs(yo - ye).max()
    if r is not None:
        assert np.array_equal(dev_to_words(ro), ero)
    if c["dtype"] == "f16":   # the reference's python golden (5e-3 in its own test)
        idx = golden[f"rms/{name}/out/idx"]
        g = golden[f"rms/{name}/out/val"]
        assert np.all(np.abs(yo.reshape(-1)[idx] - g) <= 2 * _ulp(g, "f16") + 1e-7)


def test_rms_norm_torch_binding_and_library_op():
    import tecoops
    c = cases.RMS_CASES["api_add_4096"]
    x, w, r = cases.rms_inputs(c)
    ref_out, ref_ro = _run_capi(c, x, w, r)
    from gpu_util import words_to_dev
    dx, dw, dr = (words_to_dev(a, "f16") for a in (x, w, r))
    out, ro = torch.empty_like(dx), torch.empty_like(dx)
    tecoops.rms_norm(dx, dw, dr, out, ro, c["eps"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(ro, ref_ro)
    out2 = torch.empty_like(dx)
    torch.ops.tecoops.rms_norm(dx, dw, None, out2, None, c["eps"])
    torch.cuda.synchronize()
    c2 = dict(c, res=False)
    ref2, _ = _run_capi(c2, x, w, None)
    assert torch.equal(out2, ref2)


def test_rms_norm_plugins():
    """plugin_rms_norm / plugin_rms_norm_add through the stand-in engine host."""
    from gpu_util import words_to_dev
    from tecoops import plugin
    c = cases.RMS_CASES["zoo3"]
    x, w, r = cases.rms_inputs(c)
    assert plugin.infer_output_shape("plugin_rms_norm_add", [[64, 2048], [2048], [64, 2048]],
                                     {"eps": c["eps"]}, n_out=2) == [[64, 2048], [64, 2048]]
    dx, dw, dr = (words_to_dev(a, "f16") for a in (x, w, r))
    out, ro = torch.empty_like(dx), torch.empty_like(dx)
    stream = torch.cuda.current_stream().cuda_stream
    plugin.enqueue("plugin_rms_norm_add", {"input": (dx.data_ptr(), [64, 2048]),
                                           "weight": (dw.data_ptr(), [2048]),
                                           "residual": (dr.data_ptr(), [64, 2048])},
                   [out.data_ptr(), ro.data_ptr()], {"eps": c["eps"]}, stream)
    ref_out, ref_ro = _run_capi(c, x, w, r)
    assert torch.equal(out, ref_out) and torch.equal(ro, ref_ro)
    out1 = torch.empty_like(dx)
    plugin.enqueue("plugin_rms_norm", {"input": (dx.data_ptr(), [64, 2048]),
                                       "weight": (dw.data_ptr(), [2048])},
                   [out1.data_ptr()], {"eps": c["eps"]}, stream)
    ref1, _ = _run_capi(dict(c, res=False), x, w, None)
    torch.cuda.synchronize()
    assert torch.equal(out1, ref1)
