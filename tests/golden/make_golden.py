"""Generate golden vectors by running the reference implementation itself.

Run where a checkout of the reference is present (it is read, never modified);
its location comes from ``--reference`` or the ``RTR_REFERENCE`` environment
variable::

    python tests/golden/make_golden.py --reference <checkout>
    python tests/golden/make_golden.py --reference <checkout> --cohort qwen1.5b-fp32 \
        --shard 0/2 --parts <dir>        # one of two processes; then --merge

It imports ``rapidtinyrec`` from that checkout and records, for the CPU:

* ``constraints_<grammar>.npz`` - ``GpuSidConstraintTables.lookup`` answers on the
  case lists ``validate_gpu_constraints.validate`` builds (every catalog prefix
  per step, random/in-range/boundary prefixes, seed 42);
* ``processor_<grammar>.npz`` - ``GpuSidConstrainedLogitsProcessor`` on a
  ``[50, V]`` normal matrix (seed 142) per step: finite positions, their values
  and a SHA-256 of all output bits;
* ``generate_<model>.json`` / ``.npz`` - ``model.generate`` (beam 50,
  ``max_new_tokens=8``, ``length_penalty=0``) under ``PrefillOnce`` +
  ``GpuSidConstrainedLogitsProcessor`` + ``fold_decode_attention(True)``,
  unpacked as ``benchmark_inference.py:150-154`` does, plus every step's
  finite scores.

Models: the two CPU models of the reference's own tests
(``tests/test_decoding.py:37-41`` seed 42 with the ``catalog()`` grammar;
``tests/test_inference_precision.py:174-185`` seed 50111 with the 4x4x4
grammar, FP32 and BF16) and the tiny synthetic workload (all 8 users).

``--cohort WORKLOAD`` runs the same reference ``generate`` on the full-size
synthetic workloads (the 1.5B-shaped FP32 and BF16 cohorts, the 0.5B-shaped FP32
cohort, the 7B-shaped BF16 model) and writes ``cohort_<workload>.npz``: per user the ranked token ids,
beam indices, sequence and transition log-probabilities, plus fingerprints of
the weights and prompts the records were made from.  BF16 follows the
reference's ``bf16-experimental`` opt-in on the CPU: the whole model cast to
bfloat16, HF's FP32 normalisation and beam scores.  The work splits into
``--shard i/n`` processes whose part files ``--merge`` joins.
"""
from __future__ import annotations

import argparse
import collections
import hashlib
import itertools
import json
import random
import sys
import warnings
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from rapidtinyrec_b200 import configs, workload  # noqa: E402


def catalog_5x5x4():
    """``tests/test_decoding.py:17-29``."""
    constraints = collections.defaultdict(set)
    root = (1, 2, 3)
    for a in range(40, 45):
        for b in range(70, 75):
            for c in range(100, 104):
                sid = (a, b, c)
                constraints[root].add(a)
                constraints[sid[:1]].add(b)
                constraints[sid[:2]].add(c)
                constraints[sid].add(510)
                constraints[sid + (510,)].add(511)
    return {k: sorted(v) for k, v in constraints.items()}


def grammar_444():
    """``tests/test_inference_precision.py:177-184``."""
    grammar = {(1, 2, 3): [100, 101, 102, 103]}
    for a in range(100, 104):
        grammar[(a,)] = [110, 111, 112, 113]
        for b in range(110, 114):
            grammar[(a, b)] = [120, 121, 122, 123]
            for c in range(120, 124):
                grammar[(a, b, c)] = [4]
                grammar[(a, b, c, 4)] = [5]
    return grammar


REF_MODEL_A = configs.ModelConfig('ref-test-decoding', layers=2, hidden=32, heads=4, kv_heads=2,
                                  head_dim=8, intermediate=64, vocab=512, tied=False, dtype='fp32',
                                  rope_theta=10000.0, newline=510, eos=511, root=(1, 2, 3))
REF_MODEL_B = configs.ModelConfig('ref-test-precision', layers=2, hidden=96, heads=6, kv_heads=2,
                                  head_dim=16, intermediate=160, vocab=512, tied=False, dtype='fp32',
                                  rope_theta=10000.0, newline=4, eos=5, root=(1, 2, 3))


def lookup_cases(tables, constraints, vocab, rng):
    """Case lists of ``validate_gpu_constraints.validate`` (:221-234)."""
    offsets, sizes = tables.metadata['sid_offsets'], tables.metadata['sid_range_sizes']
    out = {}
    for step in range(6):
        length = 3 if step == 0 else step
        cases = [k for k in constraints if len(k) == length]
        if step == 2:
            product = list(itertools.product(range(offsets[0], offsets[0] + sizes[0]),
                                             range(offsets[1], offsets[1] + sizes[1])))
            if len(product) > 6000:
                product = rng.sample(product, 6000)
            cases += product
        cases += [tuple(rng.randrange(vocab) for _ in range(length)) for _ in range(1000)]
        if length == 3:
            cases += [tuple(offsets[j] + rng.randrange(sizes[j]) for j in range(3)) for _ in range(1000)]
        cases += [(0,) * length, (vocab - 1,) * length, (-1,) * length]
        out[step] = list(dict.fromkeys(cases))
    return out


def write_constraint_fixtures(name, constraints, root, newline, eos, vocab, ref):
    tables = ref.GpuSidConstraintTables(constraints, root, newline, eos, 'cpu')
    rng = random.Random(42)
    cases = lookup_cases(tables, constraints, vocab, rng)
    arrays = {'meta': np.array(json.dumps({'root': list(root), 'newline': newline, 'eos': eos,
                                           'vocab': vocab, 'metadata': tables.metadata}))}
    for step, rows in cases.items():
        x = torch.tensor(rows, dtype=torch.long)
        arrays[f'cases_{step}'] = x.numpy().astype(np.int32)
        arrays[f'lookup_{step}'] = tables.lookup(step, x).numpy().astype(np.int32)
        # semantic answer of the released processor for the same prefixes
        arrays[f'allowed_{step}'] = np.array([json.dumps(constraints.get(tuple(r), [eos])) for r in rows])
    np.savez_compressed(HERE / f'constraints_{name}.npz', **arrays)

    # processor bits (validate_gpu_constraints.py:244-265 with the CPU generator)
    gen = torch.Generator().manual_seed(142)
    scores = torch.randn((50, vocab), dtype=torch.float32, generator=gen)
    proc = {'scores_sha': np.array(hashlib.sha256(scores.numpy().tobytes()).hexdigest())}
    for step, rows in cases.items():
        chosen = rows[:20] + rows[-20:]
        if step in (0, 3):
            chosen.append(tuple(root))
        while len(chosen) < 50:
            chosen.append(rows[rng.randrange(len(rows))])
        x = torch.tensor(chosen[:50], dtype=torch.long)
        p = ref.GpuSidConstrainedLogitsProcessor(tables)
        p.count = step
        out = p(x, scores)
        r, c = torch.nonzero(torch.isfinite(out), as_tuple=True)
        proc[f'input_{step}'] = x.numpy().astype(np.int32)
        proc[f'rows_{step}'] = r.numpy().astype(np.int32)
        proc[f'cols_{step}'] = c.numpy().astype(np.int32)
        proc[f'vals_{step}'] = out[r, c].numpy()
        proc[f'sha_{step}'] = np.array(hashlib.sha256(out.view(torch.int32).numpy().tobytes()).hexdigest())
    np.savez_compressed(HERE / f'processor_{name}.npz', **proc)


def hf_model(cfg, weights, dtype):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    hf_cfg = Qwen2Config(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                         num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                         num_key_value_heads=cfg.kv_heads, rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_eps,
                         tie_word_embeddings=cfg.tied, max_position_embeddings=4096,
                         bos_token_id=1, eos_token_id=cfg.eos, pad_token_id=cfg.eos)
    model = Qwen2ForCausalLM(hf_cfg)
    state = {k: v for k, v in weights.items() if not (cfg.tied and k == 'lm_head.weight')}
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and set(missing) <= {'lm_head.weight'}, (missing, unexpected)
    model = model.to(dtype).eval()
    model.config._attn_implementation = 'sdpa'
    return model


def run_reference_generate(model, cfg, tables, prompt, ref):
    from transformers import GenerationConfig, LogitsProcessorList
    gen_cfg = GenerationConfig(max_new_tokens=8, num_beams=50, num_return_sequences=50, length_penalty=0.,
                               do_sample=False, pad_token_id=cfg.eos, eos_token_id=cfg.eos, bos_token_id=1,
                               use_cache=True)
    ids = torch.tensor([list(prompt)])
    with torch.inference_mode(), ref.fold_decode_attention(True), ref.PrefillOnce(model, 50):
        out = model.generate(ids, attention_mask=torch.ones_like(ids), generation_config=gen_cfg,
                             logits_processor=LogitsProcessorList([ref.GpuSidConstrainedLogitsProcessor(tables)]),
                             return_dict_in_generate=True, output_scores=True)
    L = ids.shape[1]
    trans = model.compute_transition_scores(out.sequences, out.scores, out.beam_indices, normalize_logits=False)
    record = {'prompt_tokens': L, 'prompt_token_ids': list(prompt),
              'beam_indices': out.beam_indices.tolist(),
              'score_dtypes': [str(s.dtype) for s in out.scores],
              'token_ids': out.sequences[:, L:].tolist(),
              'sequence_logp': out.sequences_scores.float().tolist(),
              'transition_logp': trans.float().tolist()}
    sparse = {}
    for t, s in enumerate(out.scores):
        r, c = torch.nonzero(torch.isfinite(s), as_tuple=True)
        sparse[f'rows_{t}'] = r.numpy().astype(np.int32)
        sparse[f'cols_{t}'] = c.numpy().astype(np.int32)
        sparse[f'vals_{t}'] = s[r, c].float().numpy()
    return record, sparse


def write_generate_fixture(name, cfg, weights, constraints, prompts, dtype, ref, store_weights):
    tables = ref.GpuSidConstraintTables(constraints, cfg.root, cfg.newline, cfg.eos, 'cpu')
    model = hf_model(cfg, weights, dtype)
    records, arrays = [], {}
    for u, prompt in enumerate(prompts):
        record, sparse = run_reference_generate(model, cfg, tables, prompt, ref)
        records.append(record)
        arrays.update({f'u{u}_{k}': v for k, v in sparse.items()})
    if store_weights:
        arrays.update({f'w:{k}': v.float().numpy() for k, v in weights.items()})
    np.savez_compressed(HERE / f'generate_{name}.npz', **arrays)
    meta = {'model': {k: (list(v) if isinstance(v, tuple) else v) for k, v in cfg.__dict__.items()},
            'dtype': str(dtype).removeprefix('torch.'), 'weights': 'stored' if store_weights else 'synthetic seed 0',
            'versions': {'torch': torch.__version__, 'transformers': __import__('transformers').__version__},
            'records': records}
    (HERE / f'generate_{name}.json').write_text(json.dumps(meta, indent=1))


def torch_init_weights(cfg, seed):
    """Default HF init under ``torch.manual_seed(seed)``, as the reference tests build them."""
    from transformers import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(seed)
    hf_cfg = Qwen2Config(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                         num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                         num_key_value_heads=cfg.kv_heads, max_position_embeddings=128,
                         bos_token_id=1, eos_token_id=cfg.eos, pad_token_id=cfg.eos)
    model = Qwen2ForCausalLM(hf_cfg)
    return {k: v.detach().clone() for k, v in model.state_dict().items()}


def prompts_fingerprint(prompts):
    h = hashlib.sha256()
    for p in prompts:
        h.update(np.asarray(p, dtype=np.int32).tobytes())
        h.update(b'|')
    return h.hexdigest()


def cohort_model(cfg, seed):
    """The workload's synthetic weights in a ``Qwen2ForCausalLM`` of the run's dtype.

    BF16 models are built tensor by tensor (fp32 values rounded to bfloat16, as
    ``model.to(torch.bfloat16)`` rounds them) so the 7B model never holds an
    fp32 copy of every weight at once.
    """
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from rapidtinyrec_b200 import _native
    dtype = torch.bfloat16 if cfg.dtype == 'bf16' else torch.float32
    hf_cfg = Qwen2Config(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                         num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                         num_key_value_heads=cfg.kv_heads, rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_eps,
                         tie_word_embeddings=cfg.tied, max_position_embeddings=4096,
                         bos_token_id=1, eos_token_id=cfg.eos, pad_token_id=cfg.eos)
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        model = Qwen2ForCausalLM(hf_cfg)
    finally:
        torch.set_default_dtype(old)
    params = dict(model.named_parameters())
    full, probe = hashlib.sha256(), hashlib.sha256()
    with torch.no_grad():
        for tid, (name, shape, scale, offset) in enumerate(workload.tensor_specs(cfg)):
            t = torch.empty(shape, dtype=torch.float32)
            _native.synth_fill(t, seed, tid, scale, offset)
            a = t.reshape(-1).numpy()
            full.update(name.encode())
            full.update(a.tobytes())
            probe.update(name.encode())
            probe.update(a[:4096].tobytes())
            params[name].copy_(t.to(dtype))
            del t
        if cfg.tied:
            assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    model = model.to(dtype).eval()
    model.config._attn_implementation = 'sdpa'
    return model, full.hexdigest(), probe.hexdigest()


COHORT_FIELDS = ('token_ids', 'beam_indices', 'sequence_logp', 'transition_logp')


def run_cohort_part(name, users_sel, parts, ref):
    """Reference ``generate`` for the selected cohort indices; one part file per user."""
    import time
    wl = configs.workload(name)
    cfg = wl.model
    items = workload.catalog_items(wl)
    cons = workload.constraint_dict(cfg, items)
    prompts = [u.prompt_token_ids for u in workload.users(wl, items, count=max(users_sel) + 1)]
    tables = ref.GpuSidConstraintTables(cons, cfg.root, cfg.newline, cfg.eos, 'cpu')
    parts.mkdir(parents=True, exist_ok=True)
    todo = [u for u in users_sel if not (parts / f'{name}_{u:05d}.json').exists()]
    if not todo:
        return
    t0 = time.perf_counter()
    model, full, probe = cohort_model(cfg, wl.weight_seed)
    (parts / f'{name}_weights.json').write_text(json.dumps({'weights_sha256': full, 'weights_probe_sha256': probe}))
    print(f'{name}: model ready in {time.perf_counter() - t0:.0f} s, {len(todo)} users to run', flush=True)
    for u in todo:
        t = time.perf_counter()
        record, _ = run_reference_generate(model, cfg, tables, prompts[u], ref)
        record = {k: record[k] for k in ('prompt_tokens', 'score_dtypes', *COHORT_FIELDS)}
        record['cohort_index'] = u
        record['elapsed_s'] = time.perf_counter() - t
        tmp = parts / f'{name}_{u:05d}.json.tmp'
        tmp.write_text(json.dumps(record))
        tmp.replace(parts / f'{name}_{u:05d}.json')
        print(f'{name} user {u} L={record["prompt_tokens"]} {record["elapsed_s"]:.1f} s', flush=True)


def merge_cohort(name, indices, parts):
    """Join the part files of the cohort users ``indices`` into ``cohort_<name>.npz``."""
    wl = configs.workload(name)
    items = workload.catalog_items(wl)
    everyone = workload.users(wl, items, count=max(indices) + 1)
    prompts = [everyone[u].prompt_token_ids for u in indices]
    recs = [json.loads((parts / f'{name}_{u:05d}.json').read_text()) for u in indices]
    fps = json.loads((parts / f'{name}_weights.json').read_text())
    assert all(r['cohort_index'] == u and r['prompt_tokens'] == len(p) for u, r, p in zip(indices, recs, prompts))
    assert all(r['score_dtypes'] == ['torch.float32'] * 5 for r in recs)
    arrays = {
        'cohort_index': np.array(indices, dtype=np.int32),
        'prompt_tokens': np.array([r['prompt_tokens'] for r in recs], dtype=np.int32),
        'token_ids': np.array([r['token_ids'] for r in recs], dtype=np.int32),
        'beam_indices': np.array([r['beam_indices'] for r in recs], dtype=np.int16),
        'sequence_logp': np.array([r['sequence_logp'] for r in recs], dtype=np.float32),
        'transition_logp': np.array([r['transition_logp'] for r in recs], dtype=np.float32),
        'elapsed_s': np.array([r['elapsed_s'] for r in recs], dtype=np.float32),
    }
    meta = {'workload': name, 'users': len(indices), 'dtype': wl.model.dtype,
            'weights': f'synthetic seed {wl.weight_seed}', **fps,
            'prompts_sha256': prompts_fingerprint(prompts),
            'driver': 'HF generate (beam 50, max_new_tokens=8, length_penalty=0) under the reference\'s '
                      'PrefillOnce + GpuSidConstrainedLogitsProcessor + fold_decode_attention(True), CPU',
            'versions': {'torch': torch.__version__, 'transformers': __import__('transformers').__version__},
            'threads': torch.get_num_threads()}
    arrays['meta'] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f'cohort_{name}.npz', **arrays)
    print('wrote', HERE / f'cohort_{name}.npz', flush=True)


def load_reference(path):
    sys.path.insert(0, str(path))
    from rapidtinyrec import gpu_constraints, shared_prefill, folded_attention
    return argparse.Namespace(GpuSidConstraintTables=gpu_constraints.GpuSidConstraintTables,
                              GpuSidConstrainedLogitsProcessor=gpu_constraints.GpuSidConstrainedLogitsProcessor,
                              PrefillOnce=shared_prefill.PrefillOnce,
                              fold_decode_attention=folded_attention.fold_decode_attention)


def main():
    import os
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--reference', type=Path, default=os.environ.get('RTR_REFERENCE'),
                    help='checkout of the reference (default: $RTR_REFERENCE)')
    ap.add_argument('--cohort', default=None, help='full-size workload to record (e.g. qwen1.5b-fp32)')
    ap.add_argument('--users', type=int, default=None, help='cohort users 0..N-1 (default: the whole cohort)')
    ap.add_argument('--indices', default=None, help='comma-separated cohort users instead of --users')
    ap.add_argument('--shard', default='0/1', help='i/n: this process runs users u with u %% n == i')
    ap.add_argument('--parts', type=Path, default=None, help='folder for per-user part files')
    ap.add_argument('--merge', action='store_true', help='join the part files into cohort_<workload>.npz')
    ap.add_argument('--threads', type=int, default=4)
    args = ap.parse_args()
    torch.set_num_threads(args.threads)
    warnings.simplefilter('ignore')

    if args.cohort:
        if args.indices:
            indices = [int(x) for x in args.indices.split(',')]
        else:
            indices = list(range(args.users or configs.workload(args.cohort).users))
        if args.parts is None:
            ap.error('--cohort needs --parts')
        if args.merge:
            merge_cohort(args.cohort, indices, args.parts)
            return
        if args.reference is None:
            ap.error('give --reference or set RTR_REFERENCE')
        i, n = (int(x) for x in args.shard.split('/'))
        run_cohort_part(args.cohort, [u for k, u in enumerate(indices) if k % n == i], args.parts,
                        load_reference(args.reference))
        return

    if args.reference is None:
        ap.error('give --reference or set RTR_REFERENCE')
    ref = load_reference(args.reference)
    wl = configs.workload('tiny')
    items = workload.catalog_items(wl)
    tiny_constraints = workload.constraint_dict(wl.model, items)
    grammars = {'test_catalog': (catalog_5x5x4(), (1, 2, 3), 510, 511, 512),
                'grammar_444': (grammar_444(), (1, 2, 3), 4, 5, 512),
                'tiny': (tiny_constraints, wl.model.root, wl.model.newline, wl.model.eos, wl.model.vocab)}
    for name, (cons, root, nl, eos, vocab) in grammars.items():
        write_constraint_fixtures(name, cons, root, nl, eos, vocab, ref)
        print('constraints', name, flush=True)

    wa = torch_init_weights(REF_MODEL_A, 42)
    write_generate_fixture('ref_decoding_fp32', REF_MODEL_A, wa, catalog_5x5x4(),
                           [[1, 7, 8, 1, 2, 3], [1, 7, 8, 9, 10, 11, 12, 13, 1, 2, 3]], torch.float32, ref, True)
    wb = torch_init_weights(REF_MODEL_B, 50111)
    for dt in (torch.float32, torch.bfloat16):
        write_generate_fixture(f'ref_precision_{str(dt)[6:]}', REF_MODEL_B, wb, grammar_444(),
                               [[40, 41, 42, 43, 1, 2, 3]], dt, ref, dt == torch.float32)
    print('reference test models', flush=True)

    tiny_w = workload.synth_weights(wl.model, seed=wl.weight_seed, backend='numpy')
    prompts = [u.prompt_token_ids for u in workload.users(wl, items)]
    write_generate_fixture('tiny_fp32', wl.model, tiny_w, tiny_constraints, prompts, torch.float32, ref, False)
    print('tiny workload', flush=True)


if __name__ == '__main__':
    main()
