"""QuantLinear as a drop-in nn.Linear (reference tests/test_quantlinear.py:37-105).

Attribution: against exact math on the same INT4 weights the kernel error must
be small next to the error the quantisation itself opens (INT4 g128 puts
~10% mean relative error on a kaiming-uniform layer's output; the kernels'
accumulation error is ~0.1% of that), plus the 5e-3 max/max gate.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import nibblegemm_b200 as ng
from oracle import c_oracle
from tests.conftest import max_rel

pytestmark = pytest.mark.gpu

IN, OUT = 256, 128


def make_layer(bias: bool, group_size: int = 128, seed: int = 0):
    torch.manual_seed(seed)
    linear = torch.nn.Linear(IN, OUT, bias=bias).cuda().half()
    return linear, ng.QuantLinear.from_linear(linear, group_size=group_size)


def exact_int4(x: torch.Tensor, ql: ng.QuantLinear) -> np.ndarray:
    return c_oracle.matmul_f32(x.cpu().numpy(), ql.qweight.cpu().numpy(), ql.scales.cpu().numpy(),
                               ql.group_size, ql.K)


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("M", [1, 8, 64])
@pytest.mark.parametrize("group_size", [64, 128])
def test_error_belongs_to_quantisation_not_to_the_kernel(bias, M, group_size):
    linear, ql = make_layer(bias, group_size)
    x = torch.randn(M, IN, device="cuda", dtype=torch.float16)
    y = ql(x)
    assert y.shape == (M, OUT) and y.dtype == torch.float16
    ref = torch.from_numpy(exact_int4(x, ql)).cuda()
    if bias:
        ref = ref + ql.bias.float()
    fp16 = linear(x).float()
    kernel_err = (y.float() - ref).abs().mean().item()
    quant_err = (ref - fp16).abs().mean().item()
    assert quant_err > 0.0
    assert kernel_err < 0.25 * quant_err
    assert max_rel(y.float().cpu().numpy(), ref.cpu().numpy()) <= 5e-3


@pytest.mark.parametrize("shape", [(1, 4, IN), (2, 8, IN), (3, 1, IN), (2, 64, IN)])
def test_3d_input_is_flattened_and_restored(shape):
    _, ql = make_layer(bias=True, seed=1)
    x = torch.randn(*shape, device="cuda", dtype=torch.float16)
    y = ql(x)
    assert y.shape == (*shape[:-1], OUT)
    flat = torch.from_numpy(exact_int4(x.reshape(-1, IN), ql)).cuda() + ql.bias.float()
    assert max_rel(y.reshape(-1, OUT).float().cpu().numpy(), flat.cpu().numpy()) <= 5e-3


def test_bias_is_added_exactly():
    _, ql = make_layer(bias=True, seed=2)
    x = torch.randn(4, IN, device="cuda", dtype=torch.float16)
    assert torch.equal(ql(x), ng.matmul(x, ql.packed()) + ql.bias)


def test_no_bias_is_a_plain_matmul():
    _, ql = make_layer(bias=False, seed=3)
    assert ql.bias is None
    x = torch.randn(4, IN, device="cuda", dtype=torch.float16)
    assert torch.equal(ql(x), ng.matmul(x, ql.packed()))


def test_from_linear_transposes_the_weight():
    linear, ql = make_layer(bias=False, seed=4)
    assert (ql.K, ql.N) == (IN, OUT)
    approx = ng.dequant(ql.packed()).float().cpu()
    truth = linear.weight.data.t().float().cpu()
    assert (approx - truth).abs().mean() < 0.25 * truth.abs().mean()


def test_state_dict_round_trip():
    _, ql = make_layer(bias=True, seed=5)
    sd = ql.state_dict()
    assert set(sd) == {"qweight", "scales", "bias"}
    ql2 = ng.QuantLinear(ng.QuantizedWeight(sd["qweight"], sd["scales"], 128, IN, OUT), sd["bias"])
    x = torch.randn(3, IN, device="cuda", dtype=torch.float16)
    assert torch.equal(ql(x), ql2(x))
