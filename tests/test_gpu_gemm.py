"""The projection GEMM kernels against a float64 product, through the C ABI
(``rtr_gemm_check``): every decode and prefill shape of the 1.5B and 0.5B
models, ragged row counts around the 64/128-row tiles, K of one and three
chunks, split-K and no split, run-to-run determinism."""
import pytest
import torch

pytestmark = pytest.mark.gpu

# tf32 split products: error relative to sum |x w| (measured 5e-8 .. 4.3e-7)
TF32X3_TOL = 1e-6


@pytest.fixture(scope='module')
def dev():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    return torch.device('cuda:0')


def operands(dev, M, N, K, seed):
    g = torch.Generator(device='cpu').manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dev)
    w = (0.03 * torch.randn(N, K, generator=g)).to(dev)
    return x, w


def rel_err(c, x, w):
    ref = x.double() @ w.double().T
    mag = x.double().abs() @ w.double().abs().T
    return ((c.double() - ref).abs() / mag.clamp_min(1e-30)).max().item()


SHAPES = [
    (50, 2048, 1536), (50, 1536, 1536), (50, 17920, 1536), (50, 1536, 8960),   # 1.5B decode
    (50, 1152, 896), (50, 896, 4864),                                             # 0.5B decode
    (237, 2048, 1536), (237, 17920, 1536), (237, 1536, 8960), (352, 1536, 1536),  # prefill
    (1, 512, 1536), (37, 1536, 1536), (64, 896, 4864), (65, 2048, 1536), (129, 1536, 1536),
    (50, 256, 96), (50, 512, 32), (50, 132, 64), (200, 4, 1536),
]


@pytest.mark.parametrize('M,N,K', SHAPES)
@pytest.mark.parametrize('kernel', [1, 2])
def test_tf32x3_kernels_match_float64(dev, M, N, K, kernel):
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, M, N, K, seed=M * 7 + N + K)
    c = _native.gemm(x, w, kernel)
    err = rel_err(c, x, w)
    assert err <= TF32X3_TOL, f'kernel {kernel} {M}x{N}x{K}: {err:.3e}'


@pytest.mark.parametrize('M,N,K', SHAPES)
def test_fp16_pair_kernel_matches_float64(dev, M, N, K):
    """The fp32 path's GEMM: 22-bit fp16 pairs, three products (measured
    2e-8 .. 7e-8 of sum |x w|, below the 3xTF32 kernels)."""
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, M, N, K, seed=M * 7 + N + K)
    err = rel_err(_native.gemm(x, w, 5), x, w)
    assert err <= TF32X3_TOL, f'fp16-pair {M}x{N}x{K}: {err:.3e}'


def test_fp16_pair_kernel_keeps_large_and_small_activations(dev):
    """Activations far from 1 (hundreds, 1e-4) stay within the tolerance: the
    pair's scale keeps them inside the fp16 range."""
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, 50, 2048, 1536, seed=11)
    x[:, ::97] *= 300.0
    x[:, 5::89] *= 1e-4
    assert rel_err(_native.gemm(x, w, 5), x, w) <= TF32X3_TOL


def test_dispatch_and_determinism(dev):
    from rapidtinyrec_b200 import _native
    for M in (50, 237):
        x, w = operands(dev, M, 2048, 1536, seed=M)
        a = _native.gemm(x, w, 0)
        b = _native.gemm(x, w, 0)
        assert torch.equal(a, b)                                  # fixed split order, no atomics
        assert torch.equal(a, _native.gemm(x, w, 5))
        c = _native.gemm(x, w, 1 if M <= 64 else 2)
        assert torch.equal(c, _native.gemm(x, w, 1 if M <= 64 else 2))


@pytest.mark.parametrize('N,K', [(1536, 8960), (2048, 1536), (256, 688)])
def test_fp16_pair_rows_agree_bitwise_in_64_and_128_row_ctas(dev, N, K):
    """Rows of a 64-row CTA equal the same rows inside a 128-row CTA (same
    split-K plan, same promotion order): a two-user batch matches batch 1."""
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, 100, N, K, seed=N + K)
    assert torch.equal(_native.gemm(x[:50].contiguous(), w, 5), _native.gemm(x, w, 5)[:50])


def test_tf32x3_persistent_lm_head_mode(dev):
    """More weight tiles than SMs with one row tile (the LM head's shape): the
    64-row 3xTF32 kernel runs persistent CTAs that walk several tiles."""
    from rapidtinyrec_b200 import _native
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    N = (sms + 3) * 128
    x, w = operands(dev, 50, N, 1536, seed=17)
    assert rel_err(_native.gemm(x, w, 1), x, w) <= TF32X3_TOL


def test_fp16_pair_lm_head_shape(dev):
    """More weight tiles than SMs with one 64-row tile (the LM head's shape,
    several waves of CTAs): within the tolerance, and the same bits as the same
    rows inside 128-row CTAs (a two-user batch)."""
    from rapidtinyrec_b200 import _native
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    N = (sms + 3) * 128
    x, w = operands(dev, 100, N, 1536, seed=19)
    c50 = _native.gemm(x[:50].contiguous(), w, 5)
    assert rel_err(c50, x[:50], w) <= TF32X3_TOL
    assert torch.equal(c50, _native.gemm(x, w, 5)[:50])


def test_64_and_128_row_kernels_agree_bitwise_up_to_64_rows(dev):
    """Both promote the tensor-core accumulator every 8 chunks in the same order."""
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, 50, 1536, 8960, seed=3)
    assert torch.equal(_native.gemm(x, w, 1), _native.gemm(x, w, 2))


@pytest.mark.parametrize('M,N,K', [(50, 256, 64), (50, 256, 192), (50, 256, 1536), (50, 256, 8960),
                                   (50, 17920, 1536), (50, 1536, 8960), (237, 2048, 1536), (100, 1536, 8960),
                                   (300, 17920, 1536), (766, 3584, 3584), (766, 3584, 18944)])
def test_bf16_kernel_within_one_bf16_ulp_of_the_rounded_product(dev, M, N, K):
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, M, N, K, seed=K + N)
    xb, wb = x.bfloat16().float(), w.bfloat16().float()
    want = (xb.double() @ wb.double().T).float().bfloat16().float()
    got = _native.gemm(x, w, 3)
    # one bf16 ulp of the result, plus the fp32 accumulation error where the sum cancels
    mag = (xb.double().abs() @ wb.double().abs().T).float()
    tol = want.abs() / 128.0 + 2e-6 * mag
    bad = ((got - want).abs() > tol).sum().item()
    assert bad == 0, f'{bad} of {got.numel()} beyond one bf16 ulp'
    assert ((got - want).abs() <= want.abs() / 128.0).float().mean().item() > 0.999


@pytest.mark.parametrize('N,K', [(2048, 1536), (1536, 8960), (17920, 1536)])
def test_bf16_64_and_128_row_kernels_agree_bitwise(dev, N, K):
    """Above 64 rows the bf16 GEMM runs 128-row CTAs; up to 128 rows they take
    the 64-row kernel's split plan and promotion order, so the rows agree bit
    for bit with a 50-row call (a two-user decode batch equals batch 1)."""
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, 100, N, K, seed=N + 7)
    both = _native.gemm(x, w, 3)
    assert torch.equal(both[:50], _native.gemm(x[:50].contiguous(), w, 3))
    assert torch.equal(both[50:], _native.gemm(x[50:].contiguous(), w, 3))


@pytest.mark.parametrize('M,N,K', [(50, 2048, 1536), (50, 1536, 8960), (237, 1536, 1536)])
def test_ffma_kernel_matches_float64(dev, M, N, K):
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, M, N, K, seed=5)
    assert rel_err(_native.gemm(x, w, 4), x, w) <= TF32X3_TOL


def test_bad_shapes_are_rejected(dev):
    from rapidtinyrec_b200 import _native
    x, w = operands(dev, 8, 6, 64, seed=1)
    with pytest.raises(_native.NativeError):
        _native.gemm(x, w, 1)                        # N not a multiple of 4
    x, w = operands(dev, 8, 8, 40, seed=1)
    with pytest.raises(_native.NativeError):
        _native.gemm(x, w, 4)                        # FFMA needs K % 32 == 0


@pytest.mark.parametrize('M,N,K', [(50, 2048, 1536), (50, 17920, 1536), (50, 1536, 8960), (237, 17920, 1536)])
def test_fp16_pair_and_tf32x3_on_realistic_statistics(dev, M, N, K):
    """Operands shaped like a real checkpoint's rather than uniform noise:
    RMSNorm weights folded into the weight columns (column scales log-uniform in
    [0.01, 50]), a tenth of the weights below the fp16 normal range (6.1e-5),
    and activation rows of RMS 1 with outlier channels of 1e3, 1e4 and 1e5.
    The outliers' products dominate each accumulation window of the tensor
    core, whose fp32 sums keep fewer bits of the small terms added to them:
    measured on B200, fp16 pairs 4.7e-7 .. 1.8e-6 of sum |x w|, 3xTF32 1.0e-6
    .. 3.4e-6 (against 2e-8 .. 7e-8 and 7e-8 .. 2.4e-7 on uniform data)."""
    from rapidtinyrec_b200 import _native
    g = torch.Generator(device='cpu').manual_seed(M + N + K)
    col = torch.exp(torch.empty(K).uniform_(float(torch.log(torch.tensor(0.01))),
                                            float(torch.log(torch.tensor(50.0))), generator=g))
    w = 0.02 * torch.randn(N, K, generator=g) * col
    tiny = torch.rand(N, K, generator=g) < 0.1
    w[tiny] = 3e-5 * torch.randn(int(tiny.sum()), generator=g)
    x = torch.randn(M, K, generator=g)
    for v, ch in ((1e3, 7), (1e4, 311), (1e5, K - 3)):
        x[:, ch] = v * torch.sign(torch.randn(M, generator=g))
    x, w = x.to(dev), w.to(dev)
    errs = {name: rel_err(_native.gemm(x, w, kern), x, w)
            for name, kern in (('fp16-pair', 5), ('3xTF32', 1 if M <= 64 else 2))}
    print(f'{M}x{N}x{K} error / sum|xw|: ' + ', '.join(f'{k} {v:.2e}' for k, v in errs.items()))
    assert errs['fp16-pair'] <= 4e-6 and errs['3xTF32'] <= 8e-6, errs
