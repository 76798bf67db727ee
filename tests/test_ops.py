"""decode_kernel.ops: the torch.library operator and the nn.Module.

CPU: the operator is registered with a fake implementation (shape and dtype
inference without running the kernel), and the module validates its inputs.
GPU: the module matches the oracle, ``torch.library.opcheck`` accepts the op,
and a three-layer stack captured in a CUDA graph replays to the eager result.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dkhelpers import MAX_ABS, make_problem, max_err, oracle_y, to_device


def test_operator_is_registered_with_a_fake_implementation():
    import decode_kernel  # noqa: F401  (registers the op)
    from torch._subclasses.fake_tensor import FakeTensorMode

    assert hasattr(torch.ops.decode_kernel, "w4a16_linear")
    with FakeTensorMode():
        x = torch.empty(3, 5, 256, dtype=torch.float16)
        packed = torch.empty(64, 32, dtype=torch.int32)
        scales = torch.empty(64, 2, dtype=torch.float16)
        y = torch.ops.decode_kernel.w4a16_linear(x, packed, scales)
        assert y.shape == (3, 5, 64) and y.dtype == torch.float16


def test_module_validates_and_refuses_cpu():
    from decode_kernel import W4A16Linear

    packed = torch.zeros(64, 32, dtype=torch.int32)
    with pytest.raises(ValueError):
        W4A16Linear(packed, torch.zeros(64, 3, dtype=torch.float16))
    with pytest.raises(ValueError):
        W4A16Linear(packed.float(), torch.zeros(64, 2, dtype=torch.float16))
    lin = W4A16Linear(packed, torch.zeros(64, 2, dtype=torch.float16))
    assert (lin.in_features, lin.out_features) == (256, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        lin(torch.zeros(1, 256, dtype=torch.float16))
    with pytest.raises(ValueError):
        W4A16Linear.from_linear(torch.nn.Linear(256, 64, bias=True))


@pytest.mark.gpu
def test_module_matches_oracle_and_opcheck(cuda_device):
    from decode_kernel import W4A16Linear

    packed, scales, x = make_problem(300, 1024, 4, seed=81, std=0.05)
    tp, ts, tx = to_device(packed, scales, x)
    layer = W4A16Linear(tp, ts)
    y = layer(tx)
    assert max_err(y, oracle_y(x, packed, scales)) < MAX_ABS
    y3 = layer(tx.reshape(2, 2, 1024))
    assert torch.equal(y3.reshape(4, 300), y)
    torch.library.opcheck(torch.ops.decode_kernel.w4a16_linear.default, (tx, tp, ts),
                          test_utils=("test_schema", "test_faketensor"))


@pytest.mark.gpu
def test_from_linear_and_graph_captured_stack(cuda_device):
    from decode_kernel import W4A16Linear

    torch.manual_seed(0)
    dims = [1024, 2048, 512, 1024]
    layers = [W4A16Linear.from_linear(torch.nn.Linear(a, b, bias=False).cuda())
              for a, b in zip(dims[:-1], dims[1:])]

    def stack(h):
        for layer in layers:
            h = layer(h)
        return h

    x = (torch.randn(2, dims[0], device="cuda") * 0.5).half()
    eager = stack(x)
    static_x = x.clone()
    stack(static_x)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_y = stack(static_x)
    for scale in (1.0, -0.5):
        static_x.copy_(x * scale)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(static_y, stack(x * scale))
    assert torch.equal(stack(x), eager)


def test_silu_mul_operator_fake_shape():
    import decode_kernel  # noqa: F401  (registers the op)
    from torch._subclasses.fake_tensor import FakeTensorMode

    assert hasattr(torch.ops.decode_kernel, "w4a16_silu_mul")
    with FakeTensorMode():
        x = torch.empty(2, 3, 256, dtype=torch.float16)
        pg = torch.empty(96, 32, dtype=torch.int32)
        sg = torch.empty(96, 2, dtype=torch.float16)
        h = torch.ops.decode_kernel.w4a16_silu_mul(x, pg, sg, pg, sg)
        assert h.shape == (2, 3, 96) and h.dtype == torch.float16


@pytest.mark.gpu
def test_silu_mul_operator_matches_unfused_and_opcheck(cuda_device):
    import torch.nn.functional as F

    from decode_kernel import gemv

    pg, sg, x = make_problem(200, 512, 3, seed=91, std=0.05)
    pu, su, _ = make_problem(200, 512, 1, seed=92, std=0.05)
    tg, tsg, tx = to_device(pg, sg, x)
    tu, tsu, _ = to_device(pu, su, x)
    h = torch.ops.decode_kernel.w4a16_silu_mul(tx.reshape(1, 3, 512), tg, tsg, tu, tsu)
    assert torch.equal(h.reshape(3, 200), F.silu(gemv(tg, tsg, tx)) * gemv(tu, tsu, tx))
    torch.library.opcheck(torch.ops.decode_kernel.w4a16_silu_mul.default, (tx, tg, tsg, tu, tsu),
                          test_utils=("test_schema", "test_faketensor"))
