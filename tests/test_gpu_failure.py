"""Failure detection on the device: a bounded pipeline wait that runs out.

Every mbarrier wait of the tensor-core GEMMs is bounded.  The test shortens
the bound and withholds the activation copies of the fp16-pair GEMM (through
``rtr_debug_wait_control``), so the waits run out without any fault: each CTA
stops issuing, drains what it issued, frees its tensor memory and sets the
timeout bit of the status word.  The request must fail with RTR_ERR_DEVICE
(the reference raises on a failed run, ``benchmark_inference.py:246``), and
the same session must then serve requests with results bit-identical to the
ones it gave before the failure.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

SHORT_WAIT = 4_000_000  # cycles, ~2 ms: far above any wait of a healthy launch


def _engine(tiny, dev):
    from rapidtinyrec_b200 import workload
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine
    cfg = tiny['cfg']
    weights = workload.synth_weights(cfg, seed=tiny['wl'].weight_seed, device=dev)
    tables = GpuSidConstraintTables(tiny['constraints'], cfg.root, cfg.newline, cfg.eos)
    return BeamEngine(cfg, weights, tables, max_prefix=128, device=0)


def test_bounded_wait_expires_and_the_session_recovers(tiny):
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    eng = _engine(tiny, 'cuda:0')
    users = tiny['users']
    before = [eng.generate(u.prompt_token_ids) for u in users[:2]]
    assert eng.report()['tensor_core_gemm'] == 2  # the fp16-pair kernels serve this session

    _native.wait_control(0, SHORT_WAIT, withhold_activation_copies=True)
    try:
        with pytest.raises(_native.NativeError) as err:
            eng.generate(users[0].prompt_token_ids)
    finally:
        _native.wait_control(0)  # default bound, copies issued again
    assert err.value.code == _native.RTR_ERR_DEVICE
    assert 'bounded pipeline wait ran out' in str(err.value)

    after = [eng.generate(u.prompt_token_ids) for u in users[:2]]
    for a, b in zip(before, after):
        for key in ('token_ids', 'beam_indices', 'sequence_logp', 'transition_logp'):
            assert a[key] == b[key], key
    eng.close()


def test_bounded_wait_expires_in_a_clustered_split_k_gemm():
    """o_proj's shape at 50 rows runs split-K in thread-block clusters: the
    aborted CTAs still take their tickets and meet their cluster peers, and
    the next launch of the same kernel is exact again."""
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    g = torch.Generator().manual_seed(11)
    x = (torch.rand((50, 1536), generator=g) - 0.5).cuda()
    w = ((torch.rand((1536, 1536), generator=g) - 0.5) * 0.04).cuda()
    want = _native.gemm(x, w, kernel=5)
    _native.wait_control(0, SHORT_WAIT, withhold_activation_copies=True)
    try:
        with pytest.raises(_native.NativeError) as err:
            _native.gemm(x, w, kernel=5)
    finally:
        _native.wait_control(0)
    assert err.value.code == _native.RTR_ERR_DEVICE
    got = _native.gemm(x, w, kernel=5)
    assert torch.equal(got, want)


@pytest.mark.parametrize('M,N,K', [(50, 1536, 1536), (100, 1536, 1536), (237, 17920, 1536)])
def test_bounded_wait_expires_in_the_bf16_gemm(M, N, K):
    """The bf16 GEMM's waits are bounded the same way: 64-row CTAs in split-K
    clusters (50 rows), 128-row CTAs in split-K clusters (100 rows) and without
    split-K (237 rows, 2 x 140 tiles).  The aborted launch reports a device
    error and the next one is exact again."""
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    g = torch.Generator().manual_seed(M + N)
    x = (torch.rand((M, K), generator=g) - 0.5).cuda()
    w = ((torch.rand((N, K), generator=g) - 0.5) * 0.04).cuda()
    want = _native.gemm(x, w, kernel=3)
    _native.wait_control(0, SHORT_WAIT, withhold_activation_copies=True)
    try:
        with pytest.raises(_native.NativeError) as err:
            _native.gemm(x, w, kernel=3)
    finally:
        _native.wait_control(0)
    assert err.value.code == _native.RTR_ERR_DEVICE
    got = _native.gemm(x, w, kernel=3)
    assert torch.equal(got, want)
