"""Batched requests (several users per decode step, M = users x 50 rows in every
projection GEMM): each user's ranking against its batch-1 result on the same
session, through the C ABI."""
import dataclasses

import pytest
import torch

from test_gpu_parity import SCORE_TOL, check_invariants, compare_records

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def cuda():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    _native.load()
    return torch.device('cuda:0')


def engine(cfg, weights, cons, max_prefix, max_users):
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine
    tables = GpuSidConstraintTables(cons, cfg.root, cfg.newline, cfg.eos)
    return BeamEngine(cfg, weights, tables, max_prefix=max_prefix, max_users=max_users)


def check_batches(eng, prompts, cfg, items, exact_upto=2, bf16=False):
    single = [eng.generate(p) for p in prompts]
    for n in range(1, eng.max_users + 1):
        got = eng.generate_batch(prompts[:n])
        for u in range(n):
            check_invariants(got[u], cfg, items)
            if n <= exact_upto:
                # the same kernels and split-K partition as batch 1: identical bits
                assert got[u] == single[u], (n, u)
            elif bf16:
                # bf16 GEMM tiles hold 64 rows: more users can change a GEMM's split-K
                # partition, and a flipped bf16 rounding moves scores by a bf16 ulp
                shared = {tuple(t) for t in got[u]['token_ids']} & {tuple(t) for t in single[u]['token_ids']}
                assert len(shared) >= 45, (n, u, len(shared))
                assert got[u]['token_ids'][0] == single[u]['token_ids'][0]
            else:
                compare_records(got[u], single[u], tol=SCORE_TOL)
    # batch-1 requests still match after batched ones
    assert eng.generate(prompts[0]) == single[0]


def test_tiny_batches_match_single_user(cuda, tiny):
    eng = engine(tiny['cfg'], tiny['weights'], tiny['constraints'], 128, max_users=4)
    check_batches(eng, [u.prompt_token_ids for u in tiny['users'][:4]], tiny['cfg'], set(tiny['items']))
    eng.close()


def test_tiny_bf16_batches_match_single_user(cuda, tiny):
    cfg = dataclasses.replace(tiny['cfg'], dtype='bf16')
    eng = engine(cfg, tiny['weights'], tiny['constraints'], 128, max_users=3)
    check_batches(eng, [u.prompt_token_ids for u in tiny['users'][4:7]], cfg, set(tiny['items']), exact_upto=1,
                  bf16=True)
    eng.close()


def test_1p5b_batches_match_single_user(cuda):
    from rapidtinyrec_b200 import configs, workload
    wl = configs.workload('qwen1.5b-fp32')
    items = workload.catalog_items(wl)
    cons = workload.constraint_dict(wl.model, items)
    users = workload.users(wl, items, count=4)
    weights = workload.synth_weights(wl.model, seed=wl.weight_seed, device='cuda')
    eng = engine(wl.model, weights, cons, wl.prompt_max, max_users=4)
    del weights
    torch.cuda.empty_cache()
    check_batches(eng, [u.prompt_token_ids for u in users], wl.model, set(items))
    eng.close()


def test_batch_contract(cuda, tiny):
    from rapidtinyrec_b200._native import RTR_ERR_ARG, NativeError
    eng = engine(tiny['cfg'], tiny['weights'], tiny['constraints'], 128, max_users=2)
    prompts = [u.prompt_token_ids for u in tiny['users'][:3]]
    with pytest.raises(NativeError) as e:
        eng.generate_batch(prompts)                  # more users than the session holds
    assert e.value.code == RTR_ERR_ARG
    with pytest.raises(NativeError) as e:
        eng.generate_batch([prompts[0], [1, 2]])     # one prompt too short
    assert e.value.code == RTR_ERR_ARG
    assert len(eng.generate_batch(prompts[:2])) == 2
    eng.close()
