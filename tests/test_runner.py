"""Host-side pieces of the drop-in runner: release loader, user selection, statistics.

The release loader is exercised on a small Qwen2 checkpoint and tokenizer
written in the reference's release layout (``Office_ckpt/`` + the Amazon
catalog + a reference manifest holding the cohort).
"""
import json

import numpy as np
import pytest

from conftest import fake_tokenizer, write_fake_release
from rapidtinyrec_b200 import release, run
from rapidtinyrec_b200.engine import weight_order
from rapidtinyrec_b200.workload import User


@pytest.fixture(scope='module')
def fake_release(tmp_path_factory):
    root = tmp_path_factory.mktemp('release')
    sids = ['<a_1><b_2><c_3>', '<a_1><b_2><c_4>', '<a_5><b_0><c_7>']
    res, vocab = write_fake_release(root, sids)
    return root, res, vocab, sids


def test_release_loader_builds_config_trie_and_weights(fake_release):
    root, res, vocab, sids = fake_release
    rel = release.load_release(root, res)
    c = rel.cfg
    assert (c.layers, c.hidden, c.heads, c.kv_heads, c.head_dim, c.intermediate, c.vocab) == (2, 64, 4, 2, 16, 96, 64)
    assert c.tied and c.rms_eps == 1e-6 and c.rope_theta == 1e6
    rootids = (vocab['### '], vocab['Response'], vocab[':\n'])
    assert c.root == rootids and c.newline == vocab['\n'] and c.eos == vocab['<eos>']
    # the trie the reference builds from the catalog (benchmark_inference.py:86-91)
    want = {}
    for s in sids:
        a, b, cc = (vocab[t] for t in ('<' + x for x in s.split('<')[1:]))
        for k, v in ((rootids, a), ((a,), b), ((a, b), cc), ((a, b, cc), c.newline), ((a, b, cc, c.newline), c.eos)):
            want.setdefault(k, set()).add(v)
    assert rel.constraints == {k: sorted(v) for k, v in want.items()}
    assert set(weight_order(c)) <= set(rel.weights)
    assert [u.cohort_index for u in rel.users] == [0, 1, 2]
    assert all(u.prompt_token_ids[-3:] == rootids for u in rel.users)
    assert rel.user_records[1]['user_id'] == 'u1'


def test_release_targets_map_sid_strings_to_tokens(fake_release):
    root, res, vocab, sids = fake_release
    targets = release.load_targets(root, res)
    for u in range(3):
        s = sids[(u + 2) % len(sids)]
        assert targets[u] == tuple(vocab[t] for t in ('<' + x for x in s.split('<')[1:]))
    tok, _ = fake_tokenizer()
    with pytest.raises(ValueError, match='three'):
        release.sid_tokens(tok, '<a_1><b_2>')


def test_release_loader_rejects_a_foreign_root(fake_release):
    root, res, vocab, _ = fake_release
    tok, _ = fake_tokenizer()
    with pytest.raises(ValueError, match='root'):
        release.catalog_constraints(tok, ['<a_1><b_2><c_3>'], vocab['<eos>'], root=(9, 9, 9))


def test_model_config_rejects_non_qwen2():
    class Cfg:
        model_type = 'llama'
    with pytest.raises(ValueError, match='qwen2'):
        release.model_config(Cfg(), 'fp32', 4, 1, (1, 2, 3))


def _users(lengths):
    return [User(i, tuple(range(n))) for i, n in enumerate(lengths)]


def test_pilot_selection_takes_two_shortest_and_two_longest():
    users = _users([10, 30, 10, 20, 30, 10, 30])
    measured, warm = run.select_users(users, full_cohort=False)
    assert [u.cohort_index for u in measured] == [0, 2, 1, 4]
    assert warm == measured


def test_full_cohort_measures_everyone_and_warms_the_extremes():
    users = _users([10, 30, 10, 20])
    measured, warm = run.select_users(users, full_cohort=True)
    assert measured == users
    assert [u.cohort_index for u in warm] == [0, 1]


def test_distribution_uses_linear_interpolation_p95():
    vals = list(np.linspace(1.0, 2.0, 21))
    d = run.distribution(vals)
    assert d['n'] == 21 and d['median_s'] == pytest.approx(1.5) and d['p95_s'] == pytest.approx(1.95)
    assert run.percentile([1.0, 2.0], 0.95) == pytest.approx(1.95)


def test_compare_reports_rank_changes():
    a = {'token_ids': [[1], [2], [3]], 'sequence_logp': [-1.0, -2.0, -3.0], 'transition_logp': [[-1.0], [-2.0], [-3.0]]}
    b = {'token_ids': [[2], [1], [4]], 'sequence_logp': [-1.5, -1.6, -3.0], 'transition_logp': [[-1.5], [-1.6], [-3.0]]}
    c = run.compare(a, b)
    assert not c['ranked_tokens_equal'] and not c['top1_equal'] and c['overlap_count'] == 2
    assert c['baseline_only'] == [[3]] and c['shared_only'] == [[4]]
    assert {(r['baseline_rank'], r['shared_rank']) for r in c['changed_ranks']} == {(1, 2), (2, 1)}
    assert c['max_abs_score_difference_common'] == pytest.approx(0.6)


def test_cli_parser_keeps_the_reference_flags():
    p = run.build_parser()
    a = p.parse_args(['folded', '--synthetic', 'tiny', '--output-root', 'o', '--full-cohort', '--precision',
                      'bf16-experimental', '--repeats', '3', '--save-full-scores'])
    assert (a.mode, a.full_cohort, a.precision, a.repeats, a.save_full_scores) == ('folded', True,
                                                                                  'bf16-experimental', 3, True)
    a = p.parse_args(['prefill', '--release-root', 'r', '--reference-results', 'g', '--dtype', 'bfloat16', '--resume'])
    assert (a.mode, a.dtype, a.resume) == ('prefill', 'bfloat16', True)
    with pytest.raises(SystemExit):
        p.parse_args(['folded', '--output-root', 'o'])  # an input source is required
