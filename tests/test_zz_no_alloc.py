"""samq_linear_static_v1, the allocation-free variant of samq_linear_v1.

Callers that cannot let the library call cudaMalloc (a framework whose caching
allocator owns the device memory, serving loops that cannot take cudaMalloc's
device synchronization, hosts that must not run out of memory mid-request) use
this entry point: it keeps the staged activation operand in a fixed device
array of the library instead of allocated scratch.  These tests call it
through the C ABI and compare it with samq_linear_v1 on two calls in a row,
which also shows that the shared array is rewritten correctly by the second
call.  The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_REL = 2e-3


@pytest.fixture(scope="module")
def samq():
    import samq as module
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    module.init(0)
    return module


def weights_matrix(rng, n, k):
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 8
    return w


def call_static(samq, w, x, m, ldx, bias, epilogue, y, ldy):
    lib = samq.library()
    stream = torch.cuda.current_stream().cuda_stream
    return lib.samq_linear_static_v1(w.handle, x.data_ptr(), m, ldx,
                                     None if bias is None else bias.data_ptr(), epilogue, y.data_ptr(), ldy,
                                     stream)


def metrics(y, ref):
    y64, r64 = y.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    cos = float(np.dot(y64, r64) / (np.linalg.norm(y64) * np.linalg.norm(r64)))
    return cos, float(np.max(np.abs(y64 - r64)) / np.max(np.abs(r64)))


def test_static_entry_point_matches_linear_on_two_calls(samq, oracle):
    rng = np.random.default_rng(2024)
    cases = [(12, 1024, 768, 300, 1), (8, 4736, 256, 97, 0)]  # (type, k, n, m, epilogue)
    for qtype, k, n, m, epilogue in cases:
        rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
        w = samq.Weights(qtype, k, n, rows)
        x = torch.from_numpy(rng.normal(0, 1, (m, k)).astype(np.float32)).cuda()
        bias = torch.from_numpy(rng.normal(0, 0.1, n).astype(np.float32)).cuda()
        y_static = torch.full((m, n), -3.0, dtype=torch.float32, device="cuda")
        assert call_static(samq, w, x, m, k, bias, epilogue, y_static, n) == 0, \
            samq.library().samq_last_error_v1()
        y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        samq.linear(w, x, m, k, bias, epilogue, y_ref, n)
        torch.cuda.synchronize()
        got, ref = y_static.cpu().numpy(), y_ref.cpu().numpy()
        cos, rel = metrics(got, ref)
        assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
        np.testing.assert_array_equal(got, ref)  # same kernels, same operand: identical
        w.close()


def test_static_entry_point_rejects_oversize(samq, oracle):
    rng = np.random.default_rng(5)
    k, n = 4736, 32
    w = samq.Weights(8, k, n, oracle.quantize(8, weights_matrix(rng, n, k)))
    m = samq.STATIC_OPERAND_ELEMENTS // k + 1
    x = torch.empty((1, 4), dtype=torch.float32, device="cuda")
    y = torch.empty((1, 32), dtype=torch.float32, device="cuda")
    rc = call_static(samq, w, x, m, k, None, 0, y, n)
    assert rc == 1 and b"SAMQ_STATIC_OPERAND_ELEMENTS" in samq.library().samq_last_error_v1()
    w.close()
