"""Loader for the reference's release layout: checkpoint, tokenizer, catalog, cohort.

The reference's runners read (``benchmark_inference.py:63-98``,
``benchmark.py:157-256``)::

    R/Office_ckpt/                                     Qwen2 checkpoint + tokenizer (HF format)
    R/Amazon/info/Office_Products_5_2016-10-2018-11.txt catalog: SID text first on each line
    G/manifest.json                                    reference results; ``users`` holds the
                                                       frozen cohort with ``prompt_token_ids``

and build the SID trie by tokenising ``'### Response:\\n' + sid + '\\n'`` plus
EOS for every catalog line (``benchmark_inference.py:86-91``).  This module does
the same and returns what ``BeamEngine`` needs: a ``ModelConfig``, the weights
in Qwen2 state-dict names, the constraint dictionary and the cohort.  The
release itself is not shipped with this repository; the loader is exercised
on a small checkpoint and tokenizer written in the same layout.
"""
from __future__ import annotations

import collections
import dataclasses
import json
import re
from pathlib import Path

from .configs import ModelConfig
from .workload import User

CHECKPOINT = 'Office_ckpt'
CATALOG = Path('Amazon/info/Office_Products_5_2016-10-2018-11.txt')
ROOT_TEXT = '### Response:\n'


@dataclasses.dataclass
class Release:
    cfg: ModelConfig
    weights: dict
    constraints: dict
    users: list          # workload.User, in cohort order
    user_records: list   # the reference's user dicts, kept for manifests


def catalog_constraints(tokenizer, lines, eos_id: int, root=None):
    """prefix -> allowed next tokens, from catalog lines (``benchmark_inference.py:86-91``).

    Raises ``ValueError`` when a line's first three tokens differ from ``root``
    (the reference asserts every prompt ends in that root).
    """
    constraints = collections.defaultdict(set)
    for line in lines:
        sid = line.split('\t')[0].strip()
        if not sid:
            continue
        ids = list(tokenizer(ROOT_TEXT + sid + '\n').input_ids) + [int(eos_id)]
        if root is not None and ids[:3] != list(root):
            raise ValueError(f'catalog line {sid!r}: root tokens {ids[:3]} differ from the prompts\' {list(root)}')
        for j in range(3, len(ids)):
            constraints[tuple(ids[:j] if j == 3 else ids[3:j])].add(ids[j])
    return {k: sorted(v) for k, v in constraints.items()}


def model_config(hf_config, dtype: str, newline: int, eos: int, root, name: str = 'release') -> ModelConfig:
    """``ModelConfig`` from a Hugging Face Qwen2 config."""
    if getattr(hf_config, 'model_type', None) != 'qwen2':
        raise ValueError(f'expected a qwen2 checkpoint, got {getattr(hf_config, "model_type", None)!r}')
    if getattr(hf_config, 'use_sliding_window', False):
        raise ValueError('sliding-window attention is not supported (the reference asserts full attention)')
    heads = hf_config.num_attention_heads
    head_dim = getattr(hf_config, 'head_dim', None) or hf_config.hidden_size // heads
    theta = getattr(hf_config, 'rope_theta', None)
    if theta is None:
        theta = (getattr(hf_config, 'rope_parameters', None) or {}).get('rope_theta', 10000.0)
    return ModelConfig(name, layers=hf_config.num_hidden_layers, hidden=hf_config.hidden_size, heads=heads,
                       kv_heads=hf_config.num_key_value_heads, head_dim=head_dim,
                       intermediate=hf_config.intermediate_size, vocab=hf_config.vocab_size,
                       tied=bool(getattr(hf_config, 'tie_word_embeddings', False)), dtype=dtype,
                       rms_eps=float(hf_config.rms_norm_eps), rope_theta=float(theta), newline=int(newline),
                       eos=int(eos), root=tuple(int(t) for t in root))


def load_release(release_root: Path, reference_results: Path, dtype: str = 'fp32') -> Release:
    """Checkpoint, tokenizer, catalog trie and cohort of one release."""
    import torch
    from transformers import AutoModelForCausalLM, AutoTokenizer
    release_root, reference_results = Path(release_root), Path(reference_results)
    ckpt = release_root / CHECKPOINT
    tok = AutoTokenizer.from_pretrained(ckpt, local_files_only=True)
    manifest = json.loads((reference_results / 'manifest.json').read_text())
    records = manifest['users']
    users = [User(int(u['cohort_index']), tuple(int(t) for t in u['prompt_token_ids'])) for u in records]
    if not users:
        raise ValueError('reference manifest holds no users')
    root = users[0].prompt_token_ids[-3:]
    if any(u.prompt_token_ids[-3:] != root for u in users):
        raise ValueError('every prompt must end in the same three-token response root')
    newline = tok.encode('\n', add_special_tokens=False)
    if len(newline) != 1:
        raise ValueError(f'the newline must be one token, got {newline}')
    constraints = catalog_constraints(tok, (release_root / CATALOG).read_text().splitlines(), tok.eos_token_id, root)
    model = AutoModelForCausalLM.from_pretrained(ckpt, torch_dtype=torch.float32, local_files_only=True)
    cfg = model_config(model.config, dtype, newline[0], tok.eos_token_id, root, name=ckpt.name)
    weights = {k: v.detach() for k, v in model.state_dict().items()}
    if cfg.tied:
        weights.pop('lm_head.weight', None)
    return Release(cfg, weights, constraints, users, records)


def sid_tokens(tokenizer, sid: str):
    """Token ids of one SID string such as ``<a_12><b_3><c_44>`` (one added token
    per code, as the reference's auditor maps them, audit_results.py:117-119)."""
    codes = re.findall(r'<[^>]+>', sid)
    ids = tokenizer.convert_tokens_to_ids(codes)
    if len(ids) != 3 or any(i is None or i == tokenizer.unk_token_id for i in ids):
        raise ValueError(f'target SID {sid!r} is not three known code tokens')
    return tuple(int(i) for i in ids)


def load_targets(release_root: Path, reference_results: Path) -> dict:
    """Held-out target SID of every cohort user (``target_sid`` in the reference
    manifest), as token triples keyed by cohort index."""
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(Path(release_root) / CHECKPOINT, local_files_only=True)
    manifest = json.loads((Path(reference_results) / 'manifest.json').read_text())
    out = {}
    for u in manifest['users']:
        if u.get('target_sid'):
            out[int(u['cohort_index'])] = sid_tokens(tok, u['target_sid'])
    return out
