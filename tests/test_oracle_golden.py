"""Pin the CPU oracle to golden vectors recorded from the reference itself.

The fixtures under tests/golden were produced by tests/golden/make_golden.py,
which runs the reference's GpuSidConstraintTables / GpuSidConstrainedLogitsProcessor
/ PrefillOnce / fold_decode_attention inside Hugging Face generate on the CPU.
The oracle must reproduce them bit for bit.
"""
import hashlib
import json
import warnings

import numpy as np
import pytest
import torch

from conftest import GOLDEN, fixture_weights, load_generate_fixture
from oracle.beam_cpu import beam_search, process_scores
from oracle.qwen2_cpu import Qwen2Oracle
from oracle.sid_tables import SidTablesOracle, semantic_allowed
from tests.golden.make_golden import REF_MODEL_A, REF_MODEL_B, grammar_444, catalog_5x5x4

GRAMMARS = ['test_catalog', 'grammar_444', 'tiny']


def grammar(name, tiny=None):
    if name == 'test_catalog':
        return catalog_5x5x4(), (1, 2, 3), 510, 511
    if name == 'grammar_444':
        return grammar_444(), (1, 2, 3), 4, 5
    cfg = tiny['cfg']
    return tiny['constraints'], cfg.root, cfg.newline, cfg.eos


@pytest.mark.parametrize('name', GRAMMARS)
def test_lookup_tables_match_reference(name, tiny):
    cons, root, nl, eos = grammar(name, tiny)
    z = np.load(GOLDEN / f'constraints_{name}.npz')
    meta = json.loads(str(z['meta']))
    oracle = SidTablesOracle(cons, root, nl, eos)
    assert oracle.offsets == meta['metadata']['sid_offsets']
    assert oracle.sizes == meta['metadata']['sid_range_sizes']
    for step in range(6):
        cases = z[f'cases_{step}'].astype(np.int64)
        got = oracle.lookup(step, cases)
        assert np.array_equal(got, z[f'lookup_{step}']), step
        # the dense lookup and the released semantic processor agree as sets
        for row, allowed, prefix in zip(got[:400], z[f'allowed_{step}'][:400], cases[:400]):
            assert set(row.tolist()) == set(json.loads(str(allowed)))
            assert set(semantic_allowed(cons, eos, step, prefix)) == set(json.loads(str(allowed)))


@pytest.mark.parametrize('name', GRAMMARS)
def test_processor_bits_match_reference(name, tiny):
    cons, root, nl, eos = grammar(name, tiny)
    vocab = json.loads(str(np.load(GOLDEN / f'constraints_{name}.npz')['meta']))['vocab']
    z = np.load(GOLDEN / f'processor_{name}.npz')
    scores = torch.randn((50, vocab), dtype=torch.float32, generator=torch.Generator().manual_seed(142))
    assert hashlib.sha256(scores.numpy().tobytes()).hexdigest() == str(z['scores_sha'])
    tables = SidTablesOracle(cons, root, nl, eos)
    for step in range(6):
        x = torch.from_numpy(z[f'input_{step}'].astype(np.int64))
        for tb in (tables, None):
            out = process_scores(scores, x, cons, eos, step, tables=tb)
            assert hashlib.sha256(out.view(torch.int32).numpy().tobytes()).hexdigest() == str(z[f'sha_{step}'])


def test_grammar_violation_rejected():
    cons = dict(catalog_5x5x4())
    cons[(40,)] = cons[(40,)] + [99]
    with pytest.raises(AssertionError, match='Unexpected SID grammar'):
        SidTablesOracle(cons, (1, 2, 3), 510, 511)


CASES = [('ref_decoding_fp32', REF_MODEL_A, catalog_5x5x4, torch.float32),
         ('ref_precision_float32', REF_MODEL_B, grammar_444, torch.float32),
         ('ref_precision_bfloat16', REF_MODEL_B, grammar_444, torch.bfloat16)]


@pytest.mark.parametrize('name,cfg,cons,dtype', CASES)
def test_oracle_generate_matches_reference(name, cfg, cons, dtype):
    meta, arrays = load_generate_fixture(name)
    weights = fixture_weights(arrays if 'w:model.norm.weight' in arrays.files
                              else load_generate_fixture('ref_precision_float32')[1])
    model = Qwen2Oracle(cfg, weights, dtype=dtype)
    for u, rec in enumerate(meta['records']):
        out = beam_search(model, rec['prompt_token_ids'], cons(), cfg.eos)
        for key in ('token_ids', 'beam_indices', 'sequence_logp', 'transition_logp', 'score_dtypes'):
            assert out[key] == rec[key], key
        assert out['steps'] == 5


def test_oracle_tiny_workload_matches_reference(tiny):
    meta, arrays = load_generate_fixture('tiny_fp32')
    model = Qwen2Oracle(tiny['cfg'], tiny['weights'])
    assert [r['prompt_token_ids'] for r in meta['records']] == [list(u.prompt_token_ids) for u in tiny['users']]
    for u, rec in enumerate(meta['records']):
        out = beam_search(model, rec['prompt_token_ids'], tiny['constraints'], tiny['cfg'].eos)
        for key in ('token_ids', 'beam_indices', 'sequence_logp', 'transition_logp'):
            assert out[key] == rec[key], (u, key)
        for t, s in enumerate(out['scores']):
            r, c = torch.nonzero(torch.isfinite(s), as_tuple=True)
            assert np.array_equal(r.numpy(), arrays[f'u{u}_rows_{t}'])
            assert np.array_equal(c.numpy(), arrays[f'u{u}_cols_{t}'])
            assert np.array_equal(s[r, c].numpy(), arrays[f'u{u}_vals_{t}'])


def test_output_invariants_on_golden(tiny):
    """Invariants the reference audits (audit_decode_pilot.py:37-48)."""
    meta, _ = load_generate_fixture('tiny_fp32')
    cfg = tiny['cfg']
    items = set(tiny['items'])
    for rec in meta['records']:
        toks = [tuple(t) for t in rec['token_ids']]
        assert len(set(toks)) == 50
        for t, seq, trans in zip(toks, rec['sequence_logp'], rec['transition_logp']):
            assert t[:3] in items and t[3] == cfg.newline and t[4] == cfg.eos
            acc = np.float32(0)
            for v in trans:
                acc = np.float32(acc + np.float32(v))
            assert acc == np.float32(seq)
        assert rec['sequence_logp'] == sorted(rec['sequence_logp'], reverse=True)


# ------------------------------------------------ full-size cohort records
COHORTS = sorted(p.stem[len('cohort_'):] for p in GOLDEN.glob('cohort_*.npz'))


@pytest.mark.parametrize('name', COHORTS)
def test_cohort_fixture_matches_this_workload_and_holds_the_output_invariants(name):
    """The reference's full-size records were made from exactly the weights and
    prompts this repository generates, and satisfy the reference's own audit
    invariants (audit_decode_pilot.py:37-48): 50 distinct catalog SIDs ending
    in newline + EOS, finite scores, sequence score = sequential FP32 sum of the
    five transitions, ranks in score order."""
    from rapidtinyrec_b200 import configs, workload
    z = np.load(GOLDEN / f'cohort_{name}.npz')
    meta = json.loads(str(z['meta']))
    wl = configs.workload(name)
    cfg = wl.model
    idx = [int(u) for u in z['cohort_index']] if 'cohort_index' in z.files else list(range(meta['users']))
    items = workload.catalog_items(wl)
    everyone = workload.users(wl, items, count=max(idx) + 1)
    h = hashlib.sha256()
    for u in idx:
        h.update(np.asarray(everyone[u].prompt_token_ids, dtype=np.int32).tobytes())
        h.update(b'|')
    assert h.hexdigest() == meta['prompts_sha256']
    probe = hashlib.sha256()
    for tid, (tname, shape, scale, offset) in enumerate(workload.tensor_specs(cfg)):
        probe.update(tname.encode())
        probe.update(workload.synth_values_numpy(wl.weight_seed, tid, min(4096, int(np.prod(shape))), scale,
                                                 offset).tobytes())
    assert probe.hexdigest() == meta['weights_probe_sha256']
    iset = set(items)
    toks, seq, trans = z['token_ids'], z['sequence_logp'], z['transition_logp']
    assert toks.shape == (len(idx), 50, 5) and list(z['prompt_tokens']) == [everyone[u].prompt_tokens for u in idx]
    for r in range(len(idx)):
        sids = [tuple(int(x) for x in t) for t in toks[r]]
        assert len(set(sids)) == 50
        assert all(s[:3] in iset and s[3] == cfg.newline and s[4] == cfg.eos for s in sids)
        assert np.all(np.isfinite(trans[r]))
        for b in range(50):
            acc = np.float32(0)
            for v in trans[r, b]:
                acc = np.float32(acc + v)
            assert acc == seq[r, b]
        assert np.all(np.diff(seq[r]) <= 0)
