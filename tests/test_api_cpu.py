"""Host-side logic of the Python operator API (no GPU): argument forwarding
and defaults of gemv / w4a16_linear (python/decode_kernel/__init__.py:32-83 of
the reference), the torch binding's checks, and that nothing falls back to the
CPU."""

from __future__ import annotations

import pytest
import torch

import decode_kernel as dk


class Recorder:
    def __init__(self):
        self.calls = []

    def w4a16_gemv(self, packed, scales, x, version, split_k, reuse, wpr):
        self.calls.append((tuple(x.shape), version, split_k, reuse, wpr))
        return torch.zeros(x.shape[0], packed.shape[0], dtype=torch.float16)


@pytest.fixture
def recorder(monkeypatch):
    import decode_kernel._cuda as ext

    rec = Recorder()
    monkeypatch.setattr(ext, "w4a16_gemv", rec.w4a16_gemv)
    return rec


def _operands(m=32, k=256, b=1):
    packed = torch.zeros(m, k // 8, dtype=torch.int32)
    scales = torch.zeros(m, k // 128, dtype=torch.float16)
    x = torch.zeros(b, k, dtype=torch.float16)
    return packed, scales, x


def test_gemv_defaults_and_1d_x(recorder):
    packed, scales, x = _operands()
    y = dk.gemv(packed, scales, x[0])
    assert y.shape == (1, 32)
    assert recorder.calls[-1] == ((1, 256), 5, 4, False, 1)


def test_w4a16_linear_defaults(recorder):
    packed, scales, x = _operands(b=3)
    dk.w4a16_linear(x, packed, scales)
    assert recorder.calls[-1] == ((3, 256), 5, 1, True, 1)  # batched -> reuse path
    dk.w4a16_linear(x[:1], packed, scales, version=4)
    assert recorder.calls[-1] == ((1, 256), 4, 4, False, 1)
    dk.w4a16_linear(x[0], packed, scales)
    assert recorder.calls[-1] == ((1, 256), 5, 1, False, 1)


def test_cuda_available_false_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert dk.cuda_available() is False


def test_no_cpu_fallback():
    # CPU tensors are rejected by the binding (bindings.cpp:12-13 message).
    packed, scales, x = _operands()
    with pytest.raises(RuntimeError, match="must be CUDA tensors"):
        dk.gemv(packed, scales, x)


@pytest.mark.parametrize("kw,msg", [
    (dict(version=7), "version must be 0..5"),
    (dict(split_k=0), "split_k must be in"),
    (dict(warps_per_row=9), "warps_per_row must be in"),
])
def test_binding_range_checks(kw, msg):
    from decode_kernel import _cuda

    packed, scales, x = _operands()
    args = dict(version=5, split_k=4, reuse_weights=False, warps_per_row=1)
    args.update(kw)
    with pytest.raises(RuntimeError):
        _cuda.w4a16_gemv(packed, scales, x, **args)
