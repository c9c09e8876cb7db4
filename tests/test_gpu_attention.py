"""The prefill attention kernels against a float64 product, through the C ABI
(``rtr_attention_check``), at prompt lengths the workloads never produce: one
token, one key chunk exactly (64), one more (65), and at the 7B length.

The causal GQA softmax(q k^T / sqrt(D)) v of one layer (the reference's
prefill SDPA, ``rapidtinyrec/benchmark_inference.py:134``; query head h reads
KV group h / (heads / kv_heads)) is computed in float64 from the same inputs
(bf16-rounded inputs for the bf16 kernels).  Measured on B200, worst over the
lengths: fp32 FFMA 2.1e-6 .. 5.1e-6, fp32 tensor core (fp16 pairs) 1.4e-6 ..
2.8e-6, bf16 both 7.8e-3 .. 8.4e-3 (the output is one bf16 rounding, 2^-9
relative, of values up to ~3).  Bounds: 1e-5 and 1.2e-2.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

# (heads, kv_heads, head_dim): the 1.5B, 0.5B, 7B and tiny shapes
SHAPES = [(12, 2, 128), (14, 2, 64), (28, 4, 128), (4, 2, 64)]
LENGTHS = [1, 2, 63, 64, 65, 130, 300]


def reference(q, k, v):
    L, H, D = q.shape
    hpg = H // k.shape[0]
    qd = q.double().permute(1, 0, 2)
    kd = k.double().repeat_interleave(hpg, dim=0)
    vd = v.double().repeat_interleave(hpg, dim=0)
    s = qd @ kd.transpose(1, 2) / math.sqrt(D)
    s.masked_fill_(torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1), float('-inf'))
    return (torch.softmax(s, dim=-1) @ vd).permute(1, 0, 2)


def operands(L, heads, kv, D, seed):
    g = torch.Generator(device='cpu').manual_seed(seed)
    q = 2.0 * torch.randn(L, heads, D, generator=g)
    k = torch.randn(kv, L, D, generator=g)
    v = torch.randn(kv, L, D, generator=g)
    return q.cuda(), k.cuda(), v.cuda()


@pytest.fixture(scope='module')
def cuda():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')


@pytest.mark.parametrize('heads,kv,D', SHAPES)
def test_fp32_prefill_attention_kernels_match_float64(cuda, heads, kv, D):
    from rapidtinyrec_b200 import _native
    worst = {0: 0.0, 1: 0.0}
    for L in LENGTHS:
        q, k, v = operands(L, heads, kv, D, seed=L * 7 + D)
        ref = reference(q, k, v)
        for kernel in (0, 1):
            err = (_native.attention(q, k, v, kernel).double() - ref).abs().max().item()
            worst[kernel] = max(worst[kernel], err)
    print(f'{heads}/{kv}/{D}: FFMA {worst[0]:.2e}, tensor core {worst[1]:.2e}')
    assert worst[0] <= 1e-5 and worst[1] <= 1e-5, worst


@pytest.mark.parametrize('heads,kv,D', SHAPES)
def test_bf16_prefill_attention_kernels_match_float64(cuda, heads, kv, D):
    from rapidtinyrec_b200 import _native
    lengths = LENGTHS + ([700, 1024] if heads == 28 else [])
    worst = {2: 0.0, 3: 0.0}
    for L in lengths:
        q, k, v = operands(L, heads, kv, D, seed=L * 11 + D)
        q, k, v = (x.bfloat16().float() for x in (q, k, v))
        ref = reference(q, k, v)
        for kernel in (2, 3):
            err = (_native.attention(q, k, v, kernel).double() - ref).abs().max().item()
            worst[kernel] = max(worst[kernel], err)
    print(f'{heads}/{kv}/{D} bf16: FFMA {worst[2]:.2e}, tensor core {worst[3]:.2e}')
    assert worst[2] <= 1.2e-2 and worst[3] <= 1.2e-2, worst


def test_bad_arguments_are_rejected(cuda):
    from rapidtinyrec_b200 import _native
    q, k, v = operands(8, 12, 2, 128, seed=1)
    with pytest.raises(_native.NativeError):
        _native.attention(q[:, :, :96].contiguous(), k[:, :, :96].contiguous(), v[:, :, :96].contiguous(), 1)
    with pytest.raises(_native.NativeError):
        _native.attention(q, k, v, 7)
