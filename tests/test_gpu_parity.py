"""CUDA path vs the oracle / the reference's golden vectors, through the C ABI.

Bars (from the reference's own acceptance rules):
* trie lookups, constraint masks, generated tokens and beam parents: bit-exact;
* FP32 scores: |delta| <= 1e-4 (sequence and transition log-probabilities);
* every emitted SID is a catalog item, 50 distinct per request, the sequence
  score equals the sequential FP32 sum of the five transitions.
"""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_generate_fixture

pytestmark = pytest.mark.gpu

SCORE_TOL = 1e-4


@pytest.fixture(scope='module')
def cuda():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    _native.load()
    return torch.device('cuda:0')


def make_engine(cfg, weights, constraints, max_prefix):
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine
    tables = GpuSidConstraintTables(constraints, cfg.root, cfg.newline, cfg.eos)
    return BeamEngine(cfg, weights, tables, max_prefix=max_prefix)


TIE_TOL = 2e-5  # reference scores closer than this are a tie under FP32 reordering


def compare_records(got, ref, tol=SCORE_TOL, tie_tol=TIE_TOL):
    """Same ranked SIDs, same beam paths, scores within ``tol``.

    Beams are matched by their SID.  Two ranks may appear swapped only when the
    reference itself scores them within ``tie_tol`` (e.g. a bit-exact FP32 tie,
    whose order torch.topk leaves unspecified); every other position must be
    identical.  Returns the largest score difference.
    """
    g = {tuple(t): i for i, t in enumerate(got['token_ids'])}
    r = {tuple(t): i for i, t in enumerate(ref['token_ids'])}
    assert set(g) == set(r), 'different top-50 SID sets'
    worst = 0.0
    for sid, ri in r.items():
        gi = g[sid]
        assert got['beam_indices'][gi] == ref['beam_indices'][ri], ('beam path', sid)
        worst = max(worst, abs(got['sequence_logp'][gi] - ref['sequence_logp'][ri]),
                    *(abs(a - b) for a, b in zip(got['transition_logp'][gi], ref['transition_logp'][ri])))
        if gi != ri:
            # the reference score at the got position must tie with this SID's reference score
            tie = abs(ref['sequence_logp'][gi] - ref['sequence_logp'][ri])
            assert tie <= tie_tol, (f'rank {ri} -> {gi} moved without a tie', tie)
    assert worst <= tol, worst
    return worst


def check_invariants(rec, cfg, items):
    toks = [tuple(t) for t in rec['token_ids']]
    assert len(set(toks)) == len(toks)
    for t, seq, trans in zip(toks, rec['sequence_logp'], rec['transition_logp']):
        assert t[:3] in items and t[3] == cfg.newline and t[4] == cfg.eos
        assert all(np.isfinite(trans))
        acc = np.float32(0)
        for v in trans:
            acc = np.float32(acc + np.float32(v))
        assert acc == np.float32(seq)
    assert rec['sequence_logp'] == sorted(rec['sequence_logp'], reverse=True)


# ------------------------------------------------------------- workload
def test_device_filler_matches_numpy(cuda):
    from rapidtinyrec_b200 import _native, workload
    t = torch.empty(300007, device=cuda)
    _native.synth_fill(t, 0, 11, 0.0346, 0.0)
    assert np.array_equal(t.cpu().numpy(), workload.synth_values_numpy(0, 11, 300007, 0.0346, 0.0))


# ------------------------------------------------------------ constraints
def grammar_engine(name, tiny):
    from rapidtinyrec_b200 import configs
    from tests.golden.make_golden import catalog_5x5x4, grammar_444
    if name == 'test_catalog':
        cons, root, nl, eos, vocab = catalog_5x5x4(), (1, 2, 3), 510, 511, 512
    elif name == 'grammar_444':
        cons, root, nl, eos, vocab = grammar_444(), (1, 2, 3), 4, 5, 512
    else:
        c = tiny['cfg']
        cons, root, nl, eos, vocab = tiny['constraints'], c.root, c.newline, c.eos, c.vocab
    cfg = configs.ModelConfig('tables', layers=1, hidden=64, heads=1, kv_heads=1, head_dim=64,
                              intermediate=64, vocab=vocab, tied=True, dtype='fp32', newline=nl, eos=eos, root=root)
    return make_engine(cfg, None, cons, max_prefix=16), cons, eos


@pytest.mark.parametrize('name', ['test_catalog', 'grammar_444', 'tiny'])
def test_lookup_bit_exact_vs_reference(cuda, tiny, name):
    eng, _, _ = grammar_engine(name, tiny)
    z = np.load(GOLDEN / f'constraints_{name}.npz')
    for step in range(6):
        cases = torch.from_numpy(z[f'cases_{step}'].astype(np.int64))
        got = eng.constraint_lookup(step, cases).cpu().numpy()
        assert np.array_equal(got, z[f'lookup_{step}']), step


@pytest.mark.parametrize('name', ['test_catalog', 'grammar_444', 'tiny'])
def test_processor_mask_exact_values_close(cuda, tiny, name):
    eng, _, _ = grammar_engine(name, tiny)
    vocab = eng.cfg.vocab
    z = np.load(GOLDEN / f'processor_{name}.npz')
    scores = torch.randn((50, vocab), dtype=torch.float32, generator=torch.Generator().manual_seed(142)).to(cuda)
    for step in range(6):
        ids = torch.from_numpy(z[f'input_{step}'].astype(np.int64)).to(cuda)
        out = torch.empty_like(scores)
        eng.constraint_process(step, ids, scores, out)
        r, c = torch.nonzero(torch.isfinite(out), as_tuple=True)
        assert np.array_equal(r.cpu().numpy(), z[f'rows_{step}'])
        assert np.array_equal(c.cpu().numpy(), z[f'cols_{step}'])
        vals = out[r, c].cpu().numpy()
        assert np.abs(vals - z[f'vals_{step}']).max() <= 4e-6, step


def test_processor_rejects_aliasing(cuda, tiny):
    from rapidtinyrec_b200._native import NativeError
    eng, _, _ = grammar_engine('test_catalog', tiny)
    x = torch.zeros((50, 512), device=cuda)
    ids = torch.ones((50, 3), dtype=torch.int64, device=cuda)
    with pytest.raises(NativeError, match='alias'):
        eng.constraint_process(0, ids, x, x)


# ------------------------------------------------------------ end to end
@pytest.fixture(scope='module')
def tiny_engine(cuda, tiny):
    return make_engine(tiny['cfg'], tiny['weights'], tiny['constraints'], max_prefix=128)


def test_tiny_generate_matches_reference_golden(tiny_engine, tiny):
    meta, _ = load_generate_fixture('tiny_fp32')
    worst = 0.0
    items = set(tiny['items'])
    for rec in meta['records']:
        got = tiny_engine.generate(rec['prompt_token_ids'])
        worst = max(worst, compare_records(got, rec))
        check_invariants(got, tiny['cfg'], items)
    print(f'tiny: max |delta score| vs reference = {worst:.3e}')


@pytest.mark.parametrize('gemm', ['tf32', 'ffma'])
def test_tiny_alternate_gemm_paths_match_reference_golden(cuda, tiny, gemm, monkeypatch):
    """The GEMM switches (RTR_GEMM=tf32: the 3xTF32 kernels; =ffma: the FP32
    FFMA kernel) give the reference's SIDs and beam paths too."""
    monkeypatch.setenv('RTR_GEMM', gemm)
    eng = make_engine(tiny['cfg'], tiny['weights'], tiny['constraints'], max_prefix=128)
    assert eng.report()['tensor_core_gemm'] == (1 if gemm == 'tf32' else 0)
    meta, _ = load_generate_fixture('tiny_fp32')
    items = set(tiny['items'])
    for rec in meta['records']:
        got = eng.generate(rec['prompt_token_ids'])
        compare_records(got, rec)
        check_invariants(got, tiny['cfg'], items)


def test_tiny_folded_decode_attention_matches_reference_golden(cuda, tiny, monkeypatch):
    """RTR_ATTN=folded: the folded cluster kernel (query heads of a KV group as
    rows, keys split over 8 CTAs, TMA staging) in place of the per-head one."""
    monkeypatch.setenv('RTR_ATTN', 'folded')
    eng = make_engine(tiny['cfg'], tiny['weights'], tiny['constraints'], max_prefix=128)
    assert eng.report()['decode_attention'] == 2
    meta, _ = load_generate_fixture('tiny_fp32')
    for rec in meta['records'][:4]:
        compare_records(eng.generate(rec['prompt_token_ids']), rec)


def test_tiny_ffma_prefill_attention_matches_reference_golden(cuda, tiny, monkeypatch):
    """RTR_PREFILL_ATTN=ffma: the FFMA prefill attention kernel in place of the
    tensor-core one (the fp32 default); the decode path is unchanged."""
    monkeypatch.setenv('RTR_PREFILL_ATTN', 'ffma')
    eng = make_engine(tiny['cfg'], tiny['weights'], tiny['constraints'], max_prefix=128)
    assert eng.report()['prefill_attention'] == 0
    meta, _ = load_generate_fixture('tiny_fp32')
    for rec in meta['records'][:4]:
        compare_records(eng.generate(rec['prompt_token_ids']), rec)


def test_tiny_tensor_core_decode_attention_matches_reference_golden(cuda, tiny, monkeypatch):
    """RTR_ATTN=tc: the tensor-core kernel (query heads of a KV group as 128
    rows, prefix keys in 64-key chunks over a cluster of 8 CTAs, QK^T and P.V
    as fp16-pair tcgen05 products, the suffix keys on the FMA pipe)."""
    monkeypatch.setenv('RTR_ATTN', 'tc')
    eng = make_engine(tiny['cfg'], tiny['weights'], tiny['constraints'], max_prefix=128)
    assert eng.report()['decode_attention'] == 1
    meta, _ = load_generate_fixture('tiny_fp32')
    for rec in meta['records'][:4]:
        compare_records(eng.generate(rec['prompt_token_ids']), rec)


def test_tiny_step_scores_match_reference(tiny_engine):
    meta, arrays = load_generate_fixture('tiny_fp32')
    for u, rec in enumerate(meta['records'][:3]):
        tiny_engine.prefill(rec['prompt_token_ids'])
        for t in range(1, 5):
            tiny_engine.decode_step(t)
        got = tiny_engine.read_results()
        compare_records(got, rec)
        for t in range(5):
            s = tiny_engine.step_scores(t)
            r, c = torch.nonzero(torch.isfinite(s), as_tuple=True)
            assert np.array_equal(r.cpu().numpy(), arrays[f'u{u}_rows_{t}'])
            assert np.array_equal(c.cpu().numpy(), arrays[f'u{u}_cols_{t}'])
            assert np.abs(s[r, c].cpu().numpy() - arrays[f'u{u}_vals_{t}']).max() <= SCORE_TOL


def test_graph_and_eager_steps_bit_identical_and_repeatable(tiny_engine, tiny):
    ids = tiny['users'][3].prompt_token_ids
    a = tiny_engine.generate(ids)
    tiny_engine.prefill(ids)
    for t in range(1, 5):
        tiny_engine.decode_step(t)
    b = tiny_engine.read_results()
    c = tiny_engine.generate(tiny['users'][5].prompt_token_ids)
    d = tiny_engine.generate(ids)
    assert a == b == d
    assert c != a


def test_report_counts_match_the_captured_graph(tiny_engine, tiny):
    """The per-request launch count the bench reports equals what runs: the
    decode graph's kernel nodes plus the eager prefill kernels."""
    tiny_engine.generate(tiny['users'][0].prompt_token_ids)
    rep = tiny_engine.report()
    cfg = tiny['cfg']
    if rep['norm_fold']:
        # embed, 5 per layer (norms folded into q/k/v and gate/up, RoPE into q/k/v),
        # LM head (final norm folded) / the prefill's final norm + GEMV
        decode, prefill = 1 + 5 * cfg.layers + 1, 1 + 5 * cfg.layers + 2
    else:
        decode = prefill = 1 + 7 * cfg.layers + 2  # embed, 7 per layer (RoPE fused), final norm, LM head
    tail0 = 4   # step 0 after the prefill's GEMV: max, two sums, beam selection
    tail = 2    # decode steps: the LM head leaves the first pass's partials; second sum, selection
    assert rep['graph_kernel_nodes'] == 4 * (decode + tail) + 1   # decode steps 1-4, finalize
    assert rep['launches_per_request'] == 1 + prefill + tail0 + rep['graph_kernel_nodes']
    assert rep['tensor_core_gemm'] == 2 and rep['norm_fold'] == 1


def test_contract_violations_raise(tiny_engine, tiny):
    from rapidtinyrec_b200._native import RTR_ERR_ARG, RTR_ERR_STATE, NativeError
    with pytest.raises(NativeError) as e:
        tiny_engine.generate(list(range(1000, 1000 + 200)))
    assert e.value.code == RTR_ERR_ARG and 'capacity' in str(e.value)
    with pytest.raises(NativeError) as e:
        tiny_engine.generate([1, 2])
    assert e.value.code == RTR_ERR_ARG
    tiny_engine.prefill(tiny['users'][0].prompt_token_ids)
    with pytest.raises(NativeError) as e:
        tiny_engine.decode_step(2)
    assert e.value.code == RTR_ERR_STATE
    with pytest.raises(NativeError) as e:
        tiny_engine.read_results()
    assert e.value.code == RTR_ERR_STATE


def test_out_of_vocab_prompt_token_reported(tiny_engine, tiny):
    from rapidtinyrec_b200._native import RTR_ERR_DEVICE, NativeError
    ids = list(tiny['users'][0].prompt_token_ids)
    ids[5] = tiny['cfg'].vocab + 7
    with pytest.raises(NativeError) as e:
        tiny_engine.generate(ids)
    assert e.value.code == RTR_ERR_DEVICE
    # the session stays usable after a rejected request
    rec = tiny_engine.generate(tiny['users'][0].prompt_token_ids)
    assert len(rec['token_ids']) == 50


def test_activation_beyond_the_fp16_pair_range_is_reported(cuda, tiny, monkeypatch):
    """The fp16-pair GEMM carries activations up to 16 x 65,504: a model whose
    residual stream exceeds that (here: the embedding scaled by 1e7) fails
    with RTR_ERR_DEVICE instead of returning beams, and RTR_GEMM=tf32 serves
    the same request."""
    from rapidtinyrec_b200._native import RTR_ERR_DEVICE, NativeError
    weights = dict(tiny['weights'])
    key = next(k for k in weights if 'embed' in k)
    weights[key] = weights[key] * 1e7
    eng = make_engine(tiny['cfg'], weights, tiny['constraints'], max_prefix=128)
    assert eng.report()['tensor_core_gemm'] == 2
    assert eng.report()['prefill_attention'] == 1
    with pytest.raises(NativeError) as e:
        eng.generate(tiny['users'][0].prompt_token_ids)
    assert e.value.code == RTR_ERR_DEVICE
    monkeypatch.setenv('RTR_GEMM', 'tf32')
    eng = make_engine(tiny['cfg'], weights, tiny['constraints'], max_prefix=128)
    assert len(eng.generate(tiny['users'][0].prompt_token_ids)['token_ids']) == 50


# --------------------------------------------------- full-size parity
def full_size_case(name, n_oracle, n_props, cuda):
    from oracle.beam_cpu import beam_search
    from oracle.qwen2_cpu import Qwen2Oracle
    from rapidtinyrec_b200 import configs, workload
    wl = configs.workload(name)
    cfg = wl.model
    items = workload.catalog_items(wl)
    cons = workload.constraint_dict(cfg, items)
    users = workload.users(wl, items, count=max(n_oracle, n_props))
    weights = workload.synth_weights(cfg, seed=wl.weight_seed, device='cuda')
    eng = make_engine(cfg, weights, cons, max_prefix=wl.prompt_max)
    cpu_w = {k: v.cpu() for k, v in weights.items()}
    del weights
    torch.cuda.empty_cache()
    model = Qwen2Oracle(cfg, cpu_w)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    worst = 0.0
    iset = set(items)
    for u in users[:n_props]:
        got = eng.generate(u.prompt_token_ids)
        check_invariants(got, cfg, iset)
        if u.cohort_index < n_oracle:
            ref = beam_search(model, u.prompt_token_ids, cons, cfg.eos)
            worst = max(worst, compare_records(got, ref))
    eng.close()
    return worst


def test_primary_1p5b_fp32_matches_oracle(cuda):
    worst = full_size_case('qwen1.5b-fp32', n_oracle=2, n_props=6, cuda=cuda)
    print(f'qwen1.5b-fp32: max |delta score| vs oracle = {worst:.3e}')


def test_0p5b_fp32_head_dim_64_matches_oracle(cuda):
    worst = full_size_case('qwen0.5b-fp32', n_oracle=1, n_props=4, cuda=cuda)
    print(f'qwen0.5b-fp32: max |delta score| vs oracle = {worst:.3e}')


# ------------------------------------------------------------ bf16 mode
def bf16_stats(got, ref):
    """Rank-list agreement of a bf16 request with the bf16 oracle (the
    reference's bf16-experimental model, bit-exact to its own fixture on CPU)."""
    g = {tuple(t): i for i, t in enumerate(got['token_ids'])}
    r = {tuple(t): i for i, t in enumerate(ref['token_ids'])}
    common = set(g) & set(r)
    return {'rank_list_equal': [tuple(t) for t in got['token_ids']] == [tuple(t) for t in ref['token_ids']],
            'overlap': len(common), 'top1_equal': tuple(got['token_ids'][0]) == tuple(ref['token_ids'][0]),
            'max_abs_delta': max(abs(got['sequence_logp'][g[s]] - ref['sequence_logp'][r[s]]) for s in common)}


def bf16_case(name, n_users, cuda, weight_backend='native'):
    from oracle.beam_cpu import beam_search
    from oracle.qwen2_cpu import Qwen2Oracle
    from rapidtinyrec_b200 import configs, workload
    wl = configs.workload(name)
    cfg = wl.model.with_dtype('bf16')
    items = workload.catalog_items(wl)
    cons = workload.constraint_dict(cfg, items)
    users = workload.users(wl, items, count=n_users)
    if weight_backend == 'numpy':
        weights = workload.synth_weights(cfg, seed=wl.weight_seed, backend='numpy')
    else:
        weights = workload.synth_weights(cfg, seed=wl.weight_seed, device='cuda')
    eng = make_engine(cfg, weights, cons, max_prefix=max(u.prompt_tokens for u in users))
    rep = eng.report()
    want_attn = 0 if os.environ.get('RTR_ATTN') == 'rows' else 1
    assert rep['decode_attention'] == want_attn and rep['prefill_attention'] == (
        0 if os.environ.get('RTR_PREFILL_ATTN') == 'ffma' else 1)
    cpu_w = {k: v.cpu() for k, v in weights.items()}
    del weights
    torch.cuda.empty_cache()
    model = Qwen2Oracle(cfg, cpu_w, dtype=torch.bfloat16)
    iset = set(items)
    stats = []
    for u in users:
        got = eng.generate(u.prompt_token_ids)
        check_invariants(got, cfg, iset)
        stats.append(bf16_stats(got, beam_search(model, u.prompt_token_ids, cons, cfg.eos)))
    eng.close()
    changed = sum(not s['rank_list_equal'] for s in stats)
    print(f'{name} bf16: changed rank lists {changed}/{len(stats)}, '
          f'min overlap {min(s["overlap"] for s in stats)}/50, top-1 equal {sum(s["top1_equal"] for s in stats)}, '
          f'max |delta score| {max(s["max_abs_delta"] for s in stats):.3e}')
    return stats


def test_tiny_bf16_against_the_bf16_oracle(cuda):
    stats = bf16_case('tiny', 8, cuda, weight_backend='numpy')
    assert min(s['overlap'] for s in stats) >= 25
    assert max(s['max_abs_delta'] for s in stats) <= 0.5


def test_tiny_bf16_ffma_prefill_attention_against_the_bf16_oracle(cuda, monkeypatch):
    """RTR_PREFILL_ATTN=ffma keeps the bf16 mode's FFMA prefill attention
    (the default is the tensor-core kernel)."""
    monkeypatch.setenv('RTR_PREFILL_ATTN', 'ffma')
    stats = bf16_case('tiny', 8, cuda, weight_backend='numpy')
    assert min(s['overlap'] for s in stats) >= 25
    assert max(s['max_abs_delta'] for s in stats) <= 0.5


def test_tiny_bf16_per_head_decode_attention_against_the_bf16_oracle(cuda, monkeypatch):
    """RTR_ATTN=rows keeps the bf16 mode's per-head decode attention (the
    default is the tensor-core cluster kernel)."""
    monkeypatch.setenv('RTR_ATTN', 'rows')
    stats = bf16_case('tiny', 8, cuda, weight_backend='numpy')
    assert min(s['overlap'] for s in stats) >= 25
    assert max(s['max_abs_delta'] for s in stats) <= 0.5


def test_1p5b_bf16_against_the_bf16_oracle(cuda):
    stats = bf16_case('qwen1.5b-bf16', 1, cuda)
    assert min(s['overlap'] for s in stats) >= 25
    assert max(s['max_abs_delta'] for s in stats) <= 0.5
