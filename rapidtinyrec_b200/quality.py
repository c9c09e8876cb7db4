"""Quality report of one precision against another (the reference's BF16 study).

Restates the measurements of the reference's precision results
(docs/precision-results.md:14-39) and target metrics
(rapidtinyrec/audit_results.py:117-137) over two runs of the same cohort:

* per arm, with held-out targets: SID-level HitRate@k and NDCG@k for
  k in 1, 5, 10, 20, 50 (rank = position of the target's three SID tokens
  in the 50 generated sequences);
* paired: users whose hit at k appears in one arm only, and the paired
  user-bootstrap 95 % interval of the HitRate@10 and NDCG@10 differences;
* without targets as well: full ranking lists that changed, matching rank
  positions out of users x 50, mean and minimum top-50 overlap, top-1
  agreement, and the same per prompt length (the reference's subgroup view).

Records are the per-user dicts the engine returns (``token_ids`` [50][5],
``sequence_logp`` ...), keyed by cohort index.
"""
from __future__ import annotations

import math
import statistics

import numpy as np

KS = (1, 5, 10, 20, 50)


def target_rank(record, target_tokens):
    """1-based rank of the target SID (three tokens) in a record, or None."""
    t = list(target_tokens)
    for i, tokens in enumerate(record['token_ids']):
        if list(tokens[:3]) == t:
            return i + 1
    return None


def target_metrics(ranks, ks=KS):
    n = len(ranks)
    out = {}
    for k in ks:
        hits = [r is not None and r <= k for r in ranks]
        out[str(k)] = {'hits': int(sum(hits)), 'hit_rate': sum(hits) / n if n else 0.0,
                       'ndcg': sum(1.0 / math.log2(r + 1) for r in ranks if r is not None and r <= k) / n if n else 0.0}
    return out


def _user_gain(rank, k):
    return 1.0 / math.log2(rank + 1) if rank is not None and rank <= k else 0.0


def bootstrap_interval(diffs, resamples=10000, seed=0, level=0.95):
    """Paired user bootstrap of the mean difference: (low, high)."""
    d = np.asarray(diffs, dtype=np.float64)
    if d.size == 0:
        return (0.0, 0.0)
    rng = np.random.Generator(np.random.PCG64(seed))
    idx = rng.integers(0, d.size, size=(resamples, d.size))
    means = d[idx].mean(axis=1)
    lo, hi = np.quantile(means, [(1 - level) / 2, 1 - (1 - level) / 2])
    return (float(lo), float(hi))


def ranking_agreement(control, candidate):
    """Rank-list agreement of two runs over the same users (dicts cohort -> record)."""
    users = sorted(control)
    changed = positions = top1 = 0
    overlaps = []
    for u in users:
        a = [tuple(t) for t in control[u]['token_ids']]
        b = [tuple(t) for t in candidate[u]['token_ids']]
        changed += a != b
        positions += sum(x == y for x, y in zip(a, b))
        top1 += a[0] == b[0]
        overlaps.append(len(set(a) & set(b)))
    n = len(users)
    return {'users': n, 'changed_full_ranking_lists': changed, 'matching_rank_positions': positions,
            'total_rank_positions': n * len(control[users[0]]['token_ids']) if n else 0,
            'same_top1_users': top1,
            'mean_top50_overlap': statistics.mean(overlaps) if overlaps else 0.0,
            'min_top50_overlap': min(overlaps) if overlaps else 0}


def compare(control, candidate, targets=None, lengths=None, resamples=10000, seed=0):
    """Report of ``candidate`` against ``control`` (dicts cohort index -> record).

    ``targets``: cohort index -> three target SID tokens (optional).
    ``lengths``: cohort index -> prompt tokens (optional; per-length subgroups).
    """
    if set(control) != set(candidate):
        raise ValueError('the two runs must cover the same users')
    users = sorted(control)
    report = {'agreement': ranking_agreement(control, candidate)}
    if targets is not None:
        missing = [u for u in users if u not in targets]
        if missing:
            raise ValueError(f'no target for users {missing[:5]}')
        ra = [target_rank(control[u], targets[u]) for u in users]
        rb = [target_rank(candidate[u], targets[u]) for u in users]
        report['target_sid_metrics'] = {'control': target_metrics(ra), 'candidate': target_metrics(rb)}
        report['paired_target_hit_changes'] = {
            str(k): {'control_only': sum(a is not None and a <= k and not (b is not None and b <= k) for a, b in zip(ra, rb)),
                     'candidate_only': sum(b is not None and b <= k and not (a is not None and a <= k) for a, b in zip(ra, rb))}
            for k in KS}
        hit = [float(b is not None and b <= 10) - float(a is not None and a <= 10) for a, b in zip(ra, rb)]
        ndcg = [_user_gain(b, 10) - _user_gain(a, 10) for a, b in zip(ra, rb)]
        report['paired_differences_at_10'] = {
            'hit_rate': {'mean': float(np.mean(hit)), 'bootstrap_95': bootstrap_interval(hit, resamples, seed),
                         'users_gained': int(sum(d > 0 for d in hit)), 'users_lost': int(sum(d < 0 for d in hit))},
            'ndcg': {'mean': float(np.mean(ndcg)), 'bootstrap_95': bootstrap_interval(ndcg, resamples, seed + 1),
                     'users_improved': int(sum(d > 0 for d in ndcg)), 'users_regressed': int(sum(d < 0 for d in ndcg))},
            'resamples': resamples, 'seed': seed}
    if lengths is not None:
        groups = {}
        for u in users:
            groups.setdefault(int(lengths[u]), []).append(u)
        report['by_prompt_length'] = {
            str(length): ranking_agreement({u: control[u] for u in us}, {u: candidate[u] for u in us})
            for length, us in sorted(groups.items())}
    report['scope'] = ('SID-level metrics over the given users; rank-position agreement is not a '
                       'recommendation-quality metric; intervals describe this cohort only.')
    return report
