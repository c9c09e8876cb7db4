"""Drop-in runner: ``python -m rapidtinyrec_b200.run folded|prefill|quality ...``.

Same entry points, flags and per-request output layout as the reference's
``python -m rapidtinyrec.run`` (``run.py:9-19``):

* ``folded`` (``benchmark_inference.py:38-261``): sequential beam-50 requests on
  the shared-prefix path.  Writes ``manifest.json``, ``users/{repeat}_{idx:04d}.json``
  (``{repeat, cohort_index, prompt_tokens, variant, run: {elapsed_s, beam_indices,
  score_dtypes, token_ids, sequence_logp, transition_logp}}``), ``requests.json``,
  ``setup.json``, ``summary.json`` (``latency`` = n/median/p95/min/max/mean),
  ``warmup_outputs/``, ``immutable-before.json`` / ``immutable-after.json``,
  ``policy-restoration.json`` and, with ``--save-full-scores``,
  ``full_scores/{name}_{t}.f32.gz`` (the five ``[50, V]`` FP32 processed scores).
* ``prefill`` (``benchmark.py:129-404``): one paired request per user,
  ``users/{i:04d}.json`` with ``runs.{baseline,shared}`` and a ``comparison``,
  plus ``summary.json``; ``--resume`` continues a partial run.
* ``quality`` (no reference subcommand: the measurements of the reference's BF16
  study, ``docs/precision-results.md:14-39``, and its auditor's target metrics,
  ``audit_results.py:117-137``): compares a candidate ``folded`` run with a
  control run of the same users (``quality.py``); target SIDs come from the
  reference manifest's ``target_sid`` through the release tokenizer, or from
  ``--targets``.  Needs no GPU.

Inputs: the real release (``--release-root``; the frozen cohort comes from
``--reference-results``, see ``release.py``) or a seeded synthetic workload
(``--synthetic NAME``, one of ``configs.WORKLOADS``; ``--users N`` takes the
first N users).  Everything runs on the native library; there is no CPU path.
"""
from __future__ import annotations

import argparse
import datetime
import gzip
import hashlib
import json
import math
import statistics
import sys
import time
from pathlib import Path

import numpy as np

VARIANT = 'folded_prefix_replay'
PRECISIONS = ('fp32', 'bf16-experimental')


# ------------------------------------------------------------------ output
def utc_now():
    return datetime.datetime.now(datetime.timezone.utc).isoformat()


def save(path: Path, obj):
    """Atomic JSON write (temporary file, then rename)."""
    tmp = path.with_suffix(path.suffix + '.tmp')
    tmp.write_text(json.dumps(obj, indent=2, allow_nan=False))
    tmp.replace(path)


def announce(obj):
    print(json.dumps(obj, allow_nan=False), flush=True)


def percentile(values, q):
    """Linear interpolation at index (N-1)*q of the sorted values (``benchmark.py:64-68``)."""
    ordered = sorted(values)
    pos = (len(ordered) - 1) * q
    lo, hi = math.floor(pos), math.ceil(pos)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (pos - lo)


def distribution(values):
    return {'n': len(values), 'median_s': statistics.median(values), 'p95_s': percentile(values, .95),
            'min_s': min(values), 'max_s': max(values), 'mean_s': statistics.mean(values)}


def compare(a, b):
    """Rank-list comparison of two records (the fields of ``benchmark.py:71-92``)."""
    sa = [tuple(t) for t in a['token_ids']]
    sb = [tuple(t) for t in b['token_ids']]
    if not (len(set(sa)) == len(sa) == len(set(sb)) == len(sb)):
        raise RuntimeError('Expected distinct generated SIDs')
    ma = {s: (i, a['sequence_logp'][i]) for i, s in enumerate(sa)}
    mb = {s: (i, b['sequence_logp'][i]) for i, s in enumerate(sb)}
    common = set(ma) & set(mb)
    return {'ranked_tokens_equal': sa == sb, 'same_top50_set': set(sa) == set(sb), 'overlap_count': len(common),
            'exact_rank_matches': sum(x == y for x, y in zip(sa, sb)), 'top1_equal': sa[0] == sb[0],
            'sequence_scores_equal_in_rank_order': a['sequence_logp'] == b['sequence_logp'],
            'transition_scores_equal_in_rank_order': a['transition_logp'] == b['transition_logp'],
            'max_abs_score_difference_common': max((abs(ma[s][1] - mb[s][1]) for s in common), default=None),
            'changed_ranks': [{'token_ids': list(s), 'baseline_rank': ma[s][0] + 1, 'shared_rank': mb[s][0] + 1,
                               'baseline_score': ma[s][1], 'shared_score': mb[s][1]}
                              for s in sa if s in mb and ma[s][0] != mb[s][0]],
            'baseline_only': [list(s) for s in sa if s not in mb],
            'shared_only': [list(s) for s in sb if s not in ma]}


def sha256_bytes(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def library_digest():
    from . import _native
    return sha256_bytes(Path(_native.LIB_PATH).read_bytes())


# ------------------------------------------------------------------ inputs
class Inputs:
    """Model config, weights, constraint tables and cohort for one run."""

    def __init__(self, args, dtype: str):
        import torch
        from . import configs, workload
        self.dtype = dtype
        if args.release_root is not None:
            from .release import load_release
            if args.reference_results is None:
                raise SystemExit('--release-root needs --reference-results (the frozen cohort)')
            rel = load_release(args.release_root, args.reference_results, dtype)
            self.cfg, self.weights, self.constraints = rel.cfg, rel.weights, rel.constraints
            self.users, self.records = rel.users, rel.user_records
            self.source = {'release_root': str(Path(args.release_root).resolve()),
                           'reference_results': str(Path(args.reference_results).resolve())}
        else:
            wl = configs.workload(args.synthetic)
            self.cfg = wl.model.with_dtype(dtype)
            items = workload.catalog_items(wl)
            self.constraints = workload.constraint_dict(self.cfg, items)
            self.users = workload.users(wl, items, count=args.users)
            self.records = [{'cohort_index': u.cohort_index, 'prompt_tokens': u.prompt_tokens,
                             'prompt_token_ids': list(u.prompt_token_ids)} for u in self.users]
            self.weights = workload.synth_weights(self.cfg, seed=wl.weight_seed, device='cuda')
            self.source = {'synthetic': wl.name, 'weight_seed': wl.weight_seed, 'catalog_seed': wl.catalog_seed,
                           'prompt_seed': wl.prompt_seed, 'items': wl.items}
        if args.users is not None and args.release_root is not None:
            self.users, self.records = self.users[:args.users], self.records[:args.users]
        self.max_prefix = max(u.prompt_tokens for u in self.users)
        del torch

    def engine(self):
        from .constraints import GpuSidConstraintTables
        from .engine import BeamEngine
        tables = GpuSidConstraintTables(self.constraints, self.cfg.root, self.cfg.newline, self.cfg.eos)
        return BeamEngine(self.cfg, self.weights, tables, max_prefix=self.max_prefix)

    def immutable_inventory(self, engine):
        """SHA-256 of every caller-owned tensor the run reads: weights, prompts, tables."""
        import torch
        out = {}
        for name, t in self.weights.items():
            data = t.detach().contiguous().reshape(-1).view(torch.uint8).cpu().numpy().tobytes()
            out[f'parameter:{name}'] = {'sha256': sha256_bytes(data), 'shape': list(t.shape), 'dtype': str(t.dtype)}
        for u in self.users:
            out[f'input:{u.cohort_index}'] = {'sha256': sha256_bytes(np.asarray(u.prompt_token_ids, np.int64).tobytes()),
                                              'shape': [1, u.prompt_tokens], 'dtype': 'torch.int64'}
        for name, arr in engine.tables.host_arrays().items():
            out[f'table:{name}'] = {'sha256': sha256_bytes(np.ascontiguousarray(arr).tobytes()),
                                    'shape': list(arr.shape), 'dtype': str(arr.dtype)}
        return out


def eager_record(engine, ids):
    """The per-step entry points (prefill, four decode steps, read) instead of the graph."""
    engine.prefill(ids)
    for t in range(1, 5):
        engine.decode_step(t)
    return engine.read_results()


def timed(engine, ids, graph=True):
    import torch
    torch.cuda.synchronize()
    started = time.perf_counter()
    rec = engine.generate(ids) if graph else eager_record(engine, ids)
    torch.cuda.synchronize()
    return time.perf_counter() - started, rec


def memory(engine):
    import torch
    rep = engine.report()
    return {'session_device_bytes': rep['device_bytes'], 'weight_bytes': rep['weight_bytes'],
            'allocated_bytes': torch.cuda.memory_allocated(), 'reserved_bytes': torch.cuda.memory_reserved(),
            'peak_allocated_bytes': torch.cuda.max_memory_allocated()}


# ------------------------------------------------------------------ folded
def select_users(users, full_cohort):
    """Measured users and warm-up users.

    Full cohort: every user is measured once; the shortest and longest prompt
    warm up.  Pilot (the reference's default, ``benchmark_inference.py:24-34``):
    the first two users of the shortest and of the longest prompt length, who
    also warm up.
    """
    lengths = sorted({u.prompt_tokens for u in users})
    if full_cohort:
        warm = [next(u for u in users if u.prompt_tokens == n) for n in (lengths[0], lengths[-1])]
        return users, list({u.cohort_index: u for u in warm}.values())
    picked = []
    for n in (lengths[0], lengths[-1]):
        picked += [u for u in users if u.prompt_tokens == n and u not in picked][:2]
    return picked, picked


def save_scores(engine, out: Path, name: str, retained):
    """The five processed ``[50, V]`` FP32 score tensors, gzip-compressed (mtime 0)."""
    import torch
    target = out / 'full_scores'
    target.mkdir(exist_ok=True)
    scores = [engine.step_scores(t) for t in range(5)]
    meta = []
    for t, s in enumerate(scores):
        data = s.contiguous().cpu().numpy().tobytes()
        fname = f'{name}_{t}.f32.gz'
        with (target / fname).open('xb') as raw, gzip.GzipFile(fileobj=raw, mode='wb', mtime=0) as gz:
            gz.write(data)
        meta.append({'file': fname, 'shape': list(s.shape), 'dtype': 'float32', 'bytes': len(data),
                     'sha256': sha256_bytes(data)})
    save(target / f'{name}.json', meta)
    # every score tensor handed out earlier must be unchanged (the scores are owned copies)
    for old, copies in retained:
        if any(not torch.equal(x.view(torch.int32), y.view(torch.int32)) for x, y in zip(old, copies)):
            raise RuntimeError('Previously returned full scores changed')
    retained.append((scores, tuple(s.clone() for s in scores)))


def run_folded(args):
    import torch
    precision = args.precision
    dtype = 'fp32' if precision == 'fp32' else 'bf16'
    if not 1 <= args.repeats <= 10:
        raise SystemExit('--repeats must be between 1 and 10')
    out = args.output_root
    if out.exists():
        raise SystemExit('--output-root must be a new directory')
    policy_before = {'matmul_tf32': torch.backends.cuda.matmul.allow_tf32,
                     'cudnn_tf32': torch.backends.cudnn.allow_tf32}
    try:
        _folded(args, out, precision, dtype, policy_before)
    finally:
        if out.exists():
            after = {'matmul_tf32': torch.backends.cuda.matmul.allow_tf32, 'cudnn_tf32': torch.backends.cudnn.allow_tf32}
            save(out / 'policy-restoration.json', {'before': policy_before, 'after': after,
                                                   'restored': policy_before == after})


def _folded(args, out, precision, dtype, policy):
    import torch
    inp = Inputs(args, dtype)
    users, warm_users = select_users(inp.users, args.full_cohort)
    out.mkdir(parents=True, exist_ok=False)
    (out / 'users').mkdir()
    record_of = {r['cohort_index']: r for r in inp.records}
    manifest = {'experiment': 'folded_inference_v1', 'precision': precision, 'experimental': precision != 'fp32',
                'precision_policy': policy, 'variant': VARIANT, 'repeats': 1 if args.full_cohort else args.repeats,
                'full_cohort': args.full_cohort, 'save_full_scores': args.save_full_scores,
                'attention_layout': 'folded_query_heads', 'users': [record_of[u.cohort_index] for u in users],
                'dtype': 'float32' if dtype == 'fp32' else 'bfloat16', 'tf32': False,
                'numerics': ('fp32 weights and activations, fp32-accurate tensor-core projections' if dtype == 'fp32' else
                             'bf16 weights, activations and KV (rounded where a bf16 torch model rounds), fp32 '
                             'accumulation, fp32 log-softmax and beam scores'),
                'hardware': torch.cuda.get_device_name(0), 'source': inp.source,
                'model': {'layers': inp.cfg.layers, 'hidden': inp.cfg.hidden, 'heads': inp.cfg.heads,
                          'kv_heads': inp.cfg.kv_heads, 'head_dim': inp.cfg.head_dim,
                          'intermediate': inp.cfg.intermediate, 'vocab': inp.cfg.vocab, 'tied': inp.cfg.tied},
                'engine': 'rapidtinyrec_b200 native library (tcgen05 projections, one decode graph per request)',
                'sha256': {'librtr_b200.so': library_digest()},
                'versions': {'torch': torch.__version__},
                'protocol': 'Sequential folded inference, one shared physical prefix, full-vocabulary double '
                            'normalization, beam 50, all five FP32 scores. Explicit precision chosen at session '
                            'creation. Setup excluded; per-request prompt '
                            'upload, prefill, decode graph and result read included (sync to sync).'}
    save(out / 'manifest.json', manifest)
    setup_started = time.perf_counter()
    engine = inp.engine()
    if dtype == 'fp32':  # name the projection kernel the session chose (RTR_GEMM)
        kind = {2: 'fp16-pair split operands', 1: '3xTF32 split operands', 0: 'FP32 FFMA'}
        manifest['numerics'] = ('fp32 weights and activations, tensor-core projections on '
                                + kind.get(engine.report()['tensor_core_gemm'], 'unknown operands')
                                if engine.report()['tensor_core_gemm'] else
                                'fp32 weights and activations, FP32 FFMA projections')
        save(out / 'manifest.json', manifest)
    immutable_before = inp.immutable_inventory(engine)
    save(out / 'immutable-before.json', immutable_before)
    ids_of = {u.cohort_index: list(u.prompt_token_ids) for u in inp.users}

    # warm-up: the per-step entry points and the graph path must agree bit for bit
    warm = {}
    (out / 'warmup_outputs').mkdir()
    for u in warm_users:
        for mode, graph in (('eager_steps', False), (VARIANT, True)):
            _, rec = timed(engine, ids_of[u.cohort_index], graph)
            save(out / 'warmup_outputs' / f'{u.cohort_index}_{mode}.json', rec)
            if mode == 'eager_steps':
                warm[u.cohort_index] = rec
            elif rec != warm[u.cohort_index]:
                raise RuntimeError('Graph and per-step paths disagree')
    retained = []
    for u in reversed(warm_users):
        _, rec = timed(engine, ids_of[u.cohort_index])
        save(out / 'warmup_outputs' / f'{u.cohort_index}_repeat.json', rec)
        if args.save_full_scores:
            save_scores(engine, out, f'warm_{u.cohort_index}', retained)
        if rec != warm[u.cohort_index]:
            raise RuntimeError('Mixed-length candidate instability')
    torch.cuda.synchronize()
    save(out / 'setup.json', {'combined_setup_and_warmup_s': time.perf_counter() - setup_started,
                              'replay': engine.report(), 'warmup_cohort_indices': [u.cohort_index for u in warm_users],
                              'memory': memory(engine),
                              'note': 'Setup includes weight upload, tile packing and the first graph capture.'})
    torch.cuda.reset_peak_memory_stats()

    trials = ([(0, u) for u in users] if args.full_cohort else
              [(r, u) for r in range(args.repeats) for u in (users if r % 2 == 0 else list(reversed(users)))])
    rows = []
    for repeat, u in trials:
        elapsed, rec = timed(engine, ids_of[u.cohort_index])
        if args.save_full_scores:
            save_scores(engine, out, f'{repeat}_{u.cohort_index:04d}', retained)
        row = {'repeat': repeat, 'cohort_index': u.cohort_index, 'prompt_tokens': u.prompt_tokens,
               'variant': VARIANT, 'run': {'elapsed_s': elapsed, **rec}}
        rows.append(row)
        save(out / 'users' / f'{repeat}_{u.cohort_index:04d}.json', row)
        if u.cohort_index in warm and rec != warm[u.cohort_index]:
            raise RuntimeError('Replay drifted')
        announce({'stage': 'measured', 'variant': VARIANT, 'repeat': repeat, 'cohort_index': u.cohort_index,
                  'elapsed_s': elapsed})
    save(out / 'requests.json', rows)
    immutable_after = inp.immutable_inventory(engine)
    save(out / 'immutable-after.json', immutable_after)
    if immutable_before != immutable_after:
        raise RuntimeError('Parameter/input/table values changed')
    summary = {'complete': True, 'precision': precision, 'experimental': precision != 'fp32',
               'parameters_and_inputs_unchanged': True,
               'retained_score_tensors_checked': sum(len(x) for x, _ in retained), 'measured_requests': len(rows),
               'latency': distribution([r['run']['elapsed_s'] for r in rows]), 'replay': engine.report(),
               'memory': memory(engine),
               'direct_reorder': {'suffix_bytes_gathered': engine.report()['suffix_bytes_gathered'],
                                  'note': 'parents are followed through the ancestry table; nothing is copied'}}
    save(out / 'summary.json', summary)
    announce(summary)
    engine.close()


# ----------------------------------------------------------------- prefill
def summarize(records, manifest, complete=False):
    """Run summary over paired records (the fields of ``benchmark.py:95-126``)."""
    base = distribution([r['runs']['baseline']['elapsed_s'] for r in records])
    shared = distribution([r['runs']['shared']['elapsed_s'] for r in records])
    checks = [r['comparison'] for r in records]
    return {'complete': complete, 'updated_at': utc_now(), 'completed_users': len(records),
            'planned_users': len(manifest['users']), 'manifest_sha256': manifest['manifest_sha256'],
            'baseline': base, 'shared': shared, 'median_latency_ratio': base['median_s'] / shared['median_s'],
            'p95_latency_ratio': base['p95_s'] / shared['p95_s'],
            'median_paired_speedup': statistics.median(r['runs']['baseline']['elapsed_s'] / r['runs']['shared']['elapsed_s']
                                                       for r in records),
            'all50_rankings_match_users': sum(c['ranked_tokens_equal'] for c in checks),
            'same_top50_set_users': sum(c['same_top50_set'] for c in checks),
            'same_top1_users': sum(c['top1_equal'] for c in checks),
            'same_sequence_scores_users': sum(c['sequence_scores_equal_in_rank_order'] for c in checks),
            'same_transition_scores_users': sum(c['transition_scores_equal_in_rank_order'] for c in checks),
            'matching_rank_positions': sum(c['exact_rank_matches'] for c in checks),
            'total_rank_positions': 50 * len(records),
            'mismatching_cohort_indices': [r['cohort_index'] for r in records if not r['comparison']['ranked_tokens_equal']],
            'max_abs_score_difference_common': max(c['max_abs_score_difference_common'] or 0 for c in checks),
            'latency_by_prompt_length': {
                str(n): {v: distribution([r['runs'][v]['elapsed_s'] for r in records if r['prompt_tokens'] == n])
                         for v in ('baseline', 'shared')}
                for n in sorted({r['prompt_tokens'] for r in records})}}


def run_prefill(args):
    import torch
    dtype = 'fp32' if args.dtype == 'float32' else 'bf16'
    inp = Inputs(args, dtype)
    n_users = len(inp.users)
    outdir = args.output_root.resolve() / f'shared_prefill_{n_users}_users'
    outdir.mkdir(parents=True, exist_ok=True)
    users_dir = outdir / 'users'
    users_dir.mkdir(exist_ok=True)
    if list(users_dir.glob('*.json')) and not args.resume:
        raise SystemExit('Existing results: use --resume rather than overwrite')
    manifest = {'experiment': 'shared_prefill',
                'variant_definitions': {
                    'baseline': {'shared_prefill': True, 'decode': 'per-step entry points (rtr_prefill, rtr_decode_step x4, rtr_read_results)'},
                    'shared': {'shared_prefill': True, 'decode': 'one CUDA graph for decode steps 1-4 (rtr_generate)'}},
                'hardware': torch.cuda.get_device_name(0), 'device': 'CUDA', 'dtype': args.dtype,
                'num_beams': 50, 'num_return_sequences': 50, 'length_penalty': 0.0, 'max_new_tokens': 8,
                'request_batch': 1, 'output_scores': True, 'source': inp.source, 'users': inp.records,
                'sha256': {'librtr_b200.so': library_digest()},
                'protocol': 'Warm both variants once. Then one timed request per variant per user, order '
                            'alternating by cohort index; synchronize before and after each request.',
                'p95_method': 'Linear interpolation at index (N-1)*0.95 in ascending latency order.'}
    manifest['manifest_sha256'] = sha256_bytes(json.dumps(manifest, sort_keys=True).encode())
    mpath = outdir / 'manifest.json'
    if mpath.exists():
        if json.loads(mpath.read_text()) != manifest:
            raise SystemExit('Resume manifest changed')
    else:
        save(mpath, manifest)
    records = []
    for path in sorted(users_dir.glob('*.json')):
        rec = json.loads(path.read_text())
        if rec['manifest_sha256'] != manifest['manifest_sha256'] or rec['cohort_index'] != len(records):
            raise SystemExit('Expected a contiguous completed prefix of this manifest')
        records.append(rec)
    announce({'stage': 'cohort_ready', 'distinct_users': n_users, 'already_completed': len(records),
              'manifest_sha256': manifest['manifest_sha256']})
    if len(records) < n_users:
        engine = inp.engine()
        first = list(inp.users[len(records)].prompt_token_ids)
        for graph in (False, True):
            timed(engine, first, graph)
        session_id = utc_now()
        for u in inp.users[len(records):]:
            i = u.cohort_index
            order = ['baseline', 'shared'] if i % 2 == 0 else ['shared', 'baseline']
            runs = {}
            for variant in order:
                elapsed, rec = timed(engine, list(u.prompt_token_ids), graph=variant == 'shared')
                runs[variant] = {'elapsed_s': elapsed, 'token_ids': rec['token_ids'],
                                 'sequence_logp': rec['sequence_logp'], 'transition_logp': rec['transition_logp']}
            record = {'cohort_index': i, 'prompt_tokens': u.prompt_tokens, 'order': order, 'session_id': session_id,
                      'completed_at': utc_now(), 'manifest_sha256': manifest['manifest_sha256'], 'runs': runs,
                      'comparison': compare(runs['baseline'], runs['shared'])}
            save(users_dir / f'{i:04d}.json', record)
            records.append(record)
            save(outdir / 'summary.json', summarize(records, manifest, complete=len(records) == n_users))
            announce({'stage': 'user_complete', 'completed': len(records), 'planned': n_users, 'cohort_index': i,
                      'baseline_s': runs['baseline']['elapsed_s'], 'shared_s': runs['shared']['elapsed_s'],
                      'ranked_tokens_equal': record['comparison']['ranked_tokens_equal']})
        engine.close()
    final = summarize(records, manifest, complete=True)
    save(outdir / 'summary.json', final)
    announce({'stage': 'finished', **final})


# -------------------------------------------------------------------- main
def build_parser():
    ap = argparse.ArgumentParser(prog='python -m rapidtinyrec_b200.run', description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest='mode', required=True)

    def inputs(p):
        src = p.add_mutually_exclusive_group(required=True)
        src.add_argument('--release-root', type=Path, help='release with Office_ckpt/ and the Amazon catalog')
        src.add_argument('--synthetic', help='seeded synthetic workload (tiny, qwen1.5b-fp32, qwen0.5b-fp32, ...)')
        p.add_argument('--reference-results', type=Path, help='reference results holding the frozen cohort manifest')
        p.add_argument('--users', type=int, default=None, help='use the first N users of the cohort')

    f = sub.add_parser('folded', help='sequential folded inference (benchmark_inference)')
    inputs(f)
    f.add_argument('--output-root', type=Path, required=True)
    f.add_argument('--full-cohort', action='store_true')
    f.add_argument('--precision', choices=PRECISIONS, default='fp32')
    f.add_argument('--repeats', type=int, default=2, help='pilot repetitions, alternating user order')
    f.add_argument('--save-full-scores', action='store_true',
                   help='gzip FP32 processed scores of every request, outside the latency timer')
    p = sub.add_parser('prefill', help='paired per-user benchmark (benchmark --experiment shared_prefill)')
    inputs(p)
    p.add_argument('--output-root', type=Path, default=Path('results'))
    p.add_argument('--dtype', choices=('float32', 'bfloat16'), default='float32')
    p.add_argument('--resume', action='store_true')
    q = sub.add_parser('quality', help='precision report: a candidate folded run against a control run')
    q.add_argument('--control', type=Path, required=True, help='folded output of the control (e.g. fp32)')
    q.add_argument('--candidate', type=Path, required=True, help='folded output of the candidate (e.g. bf16)')
    q.add_argument('--release-root', type=Path, help='release whose tokenizer maps the target SIDs')
    q.add_argument('--reference-results', type=Path, help='reference results whose manifest holds target_sid')
    q.add_argument('--targets', type=Path, help='JSON {cohort_index: [t1, t2, t3]} (instead of the release)')
    q.add_argument('--output', type=Path, required=True)
    q.add_argument('--resamples', type=int, default=10000, help='paired user-bootstrap resamples')
    q.add_argument('--users', type=int, default=None, help=argparse.SUPPRESS)
    return ap


def read_run(out: Path):
    """First-repeat records of a folded output, keyed by cohort index."""
    rows = json.loads((Path(out) / 'requests.json').read_text())
    recs, lengths = {}, {}
    for r in rows:
        if r['repeat'] == 0:
            recs[int(r['cohort_index'])] = r['run']
            lengths[int(r['cohort_index'])] = int(r['prompt_tokens'])
    if not recs:
        raise SystemExit(f'{out}: no first-repeat requests')
    return recs, lengths


def run_quality(args):
    """The reference's BF16-study measurements (docs/precision-results.md:14-39):
    target HitRate/NDCG per arm, paired changes with bootstrap intervals, and
    rank-list agreement, overall and per prompt length."""
    from . import quality
    control, lengths = read_run(args.control)
    candidate, _ = read_run(args.candidate)
    common = sorted(set(control) & set(candidate))
    if not common:
        raise SystemExit('the two runs share no users')
    control = {u: control[u] for u in common}
    candidate = {u: candidate[u] for u in common}
    targets = None
    if args.targets is not None:
        targets = {int(k): tuple(v) for k, v in json.loads(args.targets.read_text()).items()}
    elif args.release_root is not None:
        if args.reference_results is None:
            raise SystemExit('--release-root needs --reference-results (the manifest with target_sid)')
        from .release import load_targets
        targets = load_targets(args.release_root, args.reference_results)
    if targets is not None:
        targets = {u: targets[u] for u in common if u in targets} if all(u in targets for u in common) else None
        if targets is None:
            raise SystemExit('targets do not cover every compared user')
    report = quality.compare(control, candidate, targets, {u: lengths[u] for u in common}, resamples=args.resamples)
    report['control'] = str(Path(args.control).resolve())
    report['candidate'] = str(Path(args.candidate).resolve())
    for name, path in (('control_manifest', args.control), ('candidate_manifest', args.candidate)):
        m = Path(path) / 'manifest.json'
        if m.exists():
            man = json.loads(m.read_text())
            report[name] = {k: man.get(k) for k in ('precision', 'dtype', 'experimental', 'variant')}
    report['targets'] = 'given' if targets is not None else 'none (rank-list agreement only)'
    args.output.parent.mkdir(parents=True, exist_ok=True)
    save(args.output, report)
    announce({'quality_report': str(args.output), **report['agreement']})
    return report


def main(argv=None):
    args = build_parser().parse_args(argv)
    if args.users is not None and args.users < 1:
        raise SystemExit('--users must be positive')
    if args.mode == 'quality':  # reads finished runs: no GPU needed
        return run_quality(args)
    import torch
    if not torch.cuda.is_available():
        raise SystemExit('a CUDA GPU is required (the engine has no CPU path)')
    if args.mode == 'folded':
        run_folded(args)
    else:
        run_prefill(args)


if __name__ == '__main__':
    main(sys.argv[1:])
