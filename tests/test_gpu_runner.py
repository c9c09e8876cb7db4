"""The drop-in runner end to end on a GPU: output layout, score files, resume,
and the release loader against the CPU oracle."""
import gzip
import itertools
import json

import numpy as np
import pytest
import torch

from conftest import write_fake_release
from test_gpu_parity import SCORE_TOL, check_invariants, compare_records

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def cuda():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for -m gpu tests')
    from rapidtinyrec_b200 import _native
    _native.load()
    return torch.device('cuda:0')


def test_folded_cli_writes_the_reference_layout(cuda, tmp_path, tiny):
    from rapidtinyrec_b200 import run
    out = tmp_path / 'folded'
    run.main(['folded', '--synthetic', 'tiny', '--users', '6', '--output-root', str(out), '--repeats', '2',
              '--save-full-scores'])
    for name in ('manifest.json', 'requests.json', 'setup.json', 'summary.json', 'immutable-before.json',
                 'immutable-after.json', 'policy-restoration.json'):
        assert (out / name).exists(), name
    manifest = json.loads((out / 'manifest.json').read_text())
    assert manifest['experiment'] == 'folded_inference_v1' and manifest['variant'] == 'folded_prefix_replay'
    # the pilot: up to two users of the shortest and of the longest prompt length
    lengths = [len(u.prompt_token_ids) for u in tiny['users'][:6]]
    pilot = [u['cohort_index'] for u in manifest['users']]
    assert {lengths[i] for i in pilot} == {min(lengths), max(lengths)} and 2 <= len(pilot) <= 4
    rows = json.loads((out / 'requests.json').read_text())
    assert len(rows) == 2 * len(pilot) and sorted({r['repeat'] for r in rows}) == [0, 1]
    items = set(tiny['items'])
    for r in rows:
        f = out / 'users' / f"{r['repeat']}_{r['cohort_index']:04d}.json"
        assert json.loads(f.read_text()) == r
        assert set(r['run']) == {'elapsed_s', 'beam_indices', 'score_dtypes', 'token_ids', 'sequence_logp',
                                 'transition_logp'}
        check_invariants(r['run'], tiny['cfg'], items)
    summary = json.loads((out / 'summary.json').read_text())
    assert summary['complete'] and summary['measured_requests'] == len(rows)
    assert summary['parameters_and_inputs_unchanged']
    assert summary['latency']['n'] == len(rows) and summary['retained_score_tensors_checked'] > 0
    # the saved full scores hold every transition score at its token
    V = tiny['cfg'].vocab
    r = rows[0]
    meta = json.loads((out / 'full_scores' / f"0_{r['cohort_index']:04d}.json").read_text())
    assert len(meta) == 5
    for t, m in enumerate(meta):
        raw = gzip.decompress((out / 'full_scores' / m['file']).read_bytes())
        s = np.frombuffer(raw, dtype=np.float32).reshape(50, V)
        assert m['shape'] == [50, V] and m['bytes'] == len(raw)
        for b in range(50):
            row = r['run']['beam_indices'][b][t]
            assert s[row, r['run']['token_ids'][b][t]] == np.float32(r['run']['transition_logp'][b][t])
    assert json.loads((out / 'policy-restoration.json').read_text())['restored']


def test_folded_cli_bf16_precision(cuda, tmp_path, tiny):
    from rapidtinyrec_b200 import run
    out = tmp_path / 'bf16'
    run.main(['folded', '--synthetic', 'tiny', '--users', '4', '--output-root', str(out), '--repeats', '1',
              '--precision', 'bf16-experimental'])
    manifest = json.loads((out / 'manifest.json').read_text())
    assert manifest['precision'] == 'bf16-experimental' and manifest['experimental'] and manifest['dtype'] == 'bfloat16'
    summary = json.loads((out / 'summary.json').read_text())
    assert summary['complete'] and summary['experimental']
    for r in json.loads((out / 'requests.json').read_text()):
        check_invariants(r['run'], tiny['cfg'], set(tiny['items']))


def test_prefill_cli_pairs_eager_and_graph_and_resumes(cuda, tmp_path):
    from rapidtinyrec_b200 import run
    run.main(['prefill', '--synthetic', 'tiny', '--users', '3', '--output-root', str(tmp_path)])
    outdir = tmp_path / 'shared_prefill_3_users'
    summary = json.loads((outdir / 'summary.json').read_text())
    assert summary['complete'] and summary['completed_users'] == 3
    # the per-step entry points and the decode graph are bit-identical
    assert summary['all50_rankings_match_users'] == 3 and summary['same_sequence_scores_users'] == 3
    recs = [json.loads((outdir / 'users' / f'{i:04d}.json').read_text()) for i in range(3)]
    assert [r['order'][0] for r in recs] == ['baseline', 'shared', 'baseline']
    before = [p.stat().st_mtime_ns for p in sorted((outdir / 'users').glob('*.json'))]
    run.main(['prefill', '--synthetic', 'tiny', '--users', '3', '--output-root', str(tmp_path), '--resume'])
    assert [p.stat().st_mtime_ns for p in sorted((outdir / 'users').glob('*.json'))] == before
    with pytest.raises(SystemExit, match='resume'):
        run.main(['prefill', '--synthetic', 'tiny', '--users', '3', '--output-root', str(tmp_path)])


def test_release_path_matches_the_oracle(cuda, tmp_path):
    """A checkpoint in the release layout, loaded by the runner, gives the oracle's rank lists."""
    from oracle.beam_cpu import beam_search
    from oracle.qwen2_cpu import Qwen2Oracle
    from rapidtinyrec_b200 import release, run
    sids = [f'<a_{a}><b_{b}><c_{c}>' for a, b, c in itertools.islice(itertools.product(range(8), repeat=3), 0, 512, 6)]
    res, _ = write_fake_release(tmp_path, sids, n_users=2, hidden=128, heads=2, kv_heads=1, intermediate=128)
    out = tmp_path / 'out'
    run.main(['folded', '--release-root', str(tmp_path), '--reference-results', str(res), '--output-root', str(out),
              '--full-cohort'])
    rows = json.loads((out / 'requests.json').read_text())
    rel = release.load_release(tmp_path, res)
    model = Qwen2Oracle(rel.cfg, {k: v.float() for k, v in rel.weights.items()})
    worst = 0.0
    for r in rows:
        u = rel.users[r['cohort_index']]
        ref = beam_search(model, u.prompt_token_ids, rel.constraints, rel.cfg.eos)
        worst = max(worst, compare_records(r['run'], ref))
    assert worst <= SCORE_TOL
    print(f'release path: max |delta score| vs oracle = {worst:.3e}')


def test_quality_report_bf16_against_fp32_with_release_targets(cuda, tmp_path):
    """The reference's BF16 study on a release-layout checkpoint: two folded runs,
    then the quality report with the manifest's target SIDs."""
    from rapidtinyrec_b200 import run
    sids = [f'<a_{a}><b_{b}><c_{c}>' for a, b, c in itertools.islice(itertools.product(range(8), repeat=3), 0, 512, 6)]
    res, _ = write_fake_release(tmp_path, sids, n_users=4, hidden=128, heads=2, kv_heads=1, intermediate=128)
    outs = {}
    for prec in ('fp32', 'bf16-experimental'):
        outs[prec] = tmp_path / prec
        run.main(['folded', '--release-root', str(tmp_path), '--reference-results', str(res), '--output-root',
                  str(outs[prec]), '--full-cohort', '--repeats', '1', '--precision', prec])
    report_path = tmp_path / 'quality.json'
    run.main(['quality', '--control', str(outs['fp32']), '--candidate', str(outs['bf16-experimental']),
              '--release-root', str(tmp_path), '--reference-results', str(res), '--output', str(report_path),
              '--resamples', '500'])
    rep = json.loads(report_path.read_text())
    agr = rep['agreement']
    assert agr['users'] == 4 and agr['total_rank_positions'] == 200
    assert 0 <= agr['changed_full_ranking_lists'] <= 4 and agr['min_top50_overlap'] >= 25
    for arm in ('control', 'candidate'):
        m = rep['target_sid_metrics'][arm]
        assert m['50']['hits'] >= m['10']['hits'] >= m['1']['hits']
    assert rep['candidate_manifest']['precision'] == 'bf16-experimental'
    lo, hi = rep['paired_differences_at_10']['hit_rate']['bootstrap_95']
    assert lo <= rep['paired_differences_at_10']['hit_rate']['mean'] <= hi
