"""The precision quality report (quality.py, run.py quality) on hand-made runs."""
import json

import pytest

from rapidtinyrec_b200 import quality, run


def record(sids, score0=-10.0):
    return {'token_ids': [list(s) + [9, 8] for s in sids],
            'sequence_logp': [score0 - i for i in range(len(sids))],
            'beam_indices': [[0] * 5 for _ in sids], 'transition_logp': [[0.0] * 5 for _ in sids]}


SIDS = [(100 + i, 200 + i, 300 + i) for i in range(50)]


def test_target_rank_and_metrics():
    rec = record(SIDS)
    assert quality.target_rank(rec, SIDS[0]) == 1
    assert quality.target_rank(rec, SIDS[9]) == 10
    assert quality.target_rank(rec, (1, 2, 3)) is None
    m = quality.target_metrics([1, 10, None, 11])
    assert m['10']['hits'] == 2 and m['10']['hit_rate'] == 0.5
    assert m['1']['ndcg'] == pytest.approx(1.0 / 4)
    assert m['10']['ndcg'] == pytest.approx((1.0 + 1.0 / 3.4594316186372973) / 4)


def test_agreement_counts_changed_lists_and_positions():
    a = {0: record(SIDS), 1: record(SIDS)}
    swapped = SIDS[:]
    swapped[3], swapped[4] = swapped[4], swapped[3]
    b = {0: record(SIDS), 1: record(swapped)}
    agr = quality.ranking_agreement(a, b)
    assert agr['changed_full_ranking_lists'] == 1
    assert agr['matching_rank_positions'] == 98 and agr['total_rank_positions'] == 100
    assert agr['same_top1_users'] == 2 and agr['min_top50_overlap'] == 50


def test_bootstrap_is_seeded_and_brackets_the_mean():
    d = [0.0] * 90 + [1.0] * 5 + [-1.0] * 5
    lo, hi = quality.bootstrap_interval(d, resamples=2000, seed=3)
    assert (lo, hi) == quality.bootstrap_interval(d, resamples=2000, seed=3)
    assert lo < 0.0 < hi


def test_compare_with_targets_paired_changes():
    control = {u: record(SIDS) for u in range(4)}
    candidate = {u: record(SIDS) for u in range(4)}
    moved = SIDS[:]
    moved.insert(12, moved.pop(5))        # the target of user 2 drops from rank 6 to 13
    candidate[2] = record(moved)
    targets = {0: SIDS[0], 1: (1, 2, 3), 2: SIDS[5], 3: SIDS[40]}
    rep = quality.compare(control, candidate, targets, lengths={0: 100, 1: 100, 2: 150, 3: 150}, resamples=500)
    assert rep['target_sid_metrics']['control']['10']['hits'] == 2
    assert rep['target_sid_metrics']['candidate']['10']['hits'] == 1
    assert rep['paired_target_hit_changes']['10'] == {'control_only': 1, 'candidate_only': 0}
    assert rep['paired_differences_at_10']['hit_rate']['users_lost'] == 1
    assert rep['by_prompt_length']['150']['changed_full_ranking_lists'] == 1
    with pytest.raises(ValueError):
        quality.compare(control, {0: record(SIDS)})


def write_run(root, recs, precision):
    root.mkdir()
    rows = [{'repeat': 0, 'cohort_index': u, 'prompt_tokens': 120 + u, 'variant': 'folded_prefix_replay', 'run': r}
            for u, r in recs.items()]
    (root / 'requests.json').write_text(json.dumps(rows))
    (root / 'manifest.json').write_text(json.dumps({'precision': precision, 'dtype': precision}))


def test_quality_cli(tmp_path):
    write_run(tmp_path / 'fp32', {u: record(SIDS) for u in range(3)}, 'fp32')
    write_run(tmp_path / 'bf16', {u: record(SIDS if u else SIDS[::-1]) for u in range(3)}, 'bf16-experimental')
    (tmp_path / 'targets.json').write_text(json.dumps({str(u): list(SIDS[u]) for u in range(3)}))
    out = tmp_path / 'report' / 'quality.json'
    run.main(['quality', '--control', str(tmp_path / 'fp32'), '--candidate', str(tmp_path / 'bf16'),
              '--targets', str(tmp_path / 'targets.json'), '--output', str(out), '--resamples', '200'])
    rep = json.loads(out.read_text())
    assert rep['agreement']['changed_full_ranking_lists'] == 1
    assert rep['candidate_manifest']['precision'] == 'bf16-experimental'
    assert rep['target_sid_metrics']['control']['1']['hits'] == 1   # user 0's target is its top-1
    assert rep['target_sid_metrics']['candidate']['1']['hits'] == 0
