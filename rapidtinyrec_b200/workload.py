"""Seeded synthetic stand-ins for the MiniOneRec release: weights, catalog, users.

* Weights: a counter-based hash (splitmix64 finaliser) per tensor, mapped to a
  uniform value ``(k - 2**23) * scale * 2**-23 + offset`` with ``k`` the top 24
  hash bits.  Every step is exact or a single IEEE float32 rounding, so the
  native host filler, the CUDA filler and :func:`synth_values_numpy` produce
  bit-identical tensors.  Matrices and biases have std 0.02 (the Qwen2
  ``initializer_range``); RMSNorm weights are uniform in [0.9, 1.1].
* Catalog: ``items`` unique uniform-random SID triples over 256 codes per
  level, turned into the reference's constraint dictionary exactly as
  ``benchmark_inference.py:87-91`` builds it from the release catalog.
* Users: instruction template + seeded filler + history SID triples + the
  3-token root, the prompt layout of ``source/data.py:604-658``.
"""
from __future__ import annotations

import collections
import dataclasses

import numpy as np

from .configs import SID_CODES, SID_LEVELS, ModelConfig, Workload

MATRIX_SCALE = 0.0346   # uniform half-width giving std 0.02
NORM_SCALE = 0.1

_GOLDEN = 0x9E3779B97F4A7C15
_TENSOR_MUL = 0xD1B54A32D192ED03
_MASK64 = (1 << 64) - 1


def tensor_specs(cfg: ModelConfig):
    """Canonical (name, shape, scale, offset) list; the index is the hash stream id.

    Names follow the Hugging Face Qwen2 state dict so the same tensors load into
    ``Qwen2ForCausalLM`` for the reference run.
    """
    h, q, kv, i = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.intermediate
    specs = [('model.embed_tokens.weight', (cfg.vocab, h), MATRIX_SCALE, 0.0)]
    for n in range(cfg.layers):
        p = f'model.layers.{n}.'
        specs += [
            (p + 'self_attn.q_proj.weight', (q, h), MATRIX_SCALE, 0.0),
            (p + 'self_attn.q_proj.bias', (q,), MATRIX_SCALE, 0.0),
            (p + 'self_attn.k_proj.weight', (kv, h), MATRIX_SCALE, 0.0),
            (p + 'self_attn.k_proj.bias', (kv,), MATRIX_SCALE, 0.0),
            (p + 'self_attn.v_proj.weight', (kv, h), MATRIX_SCALE, 0.0),
            (p + 'self_attn.v_proj.bias', (kv,), MATRIX_SCALE, 0.0),
            (p + 'self_attn.o_proj.weight', (h, q), MATRIX_SCALE, 0.0),
            (p + 'mlp.gate_proj.weight', (i, h), MATRIX_SCALE, 0.0),
            (p + 'mlp.up_proj.weight', (i, h), MATRIX_SCALE, 0.0),
            (p + 'mlp.down_proj.weight', (h, i), MATRIX_SCALE, 0.0),
            (p + 'input_layernorm.weight', (h,), NORM_SCALE, 1.0),
            (p + 'post_attention_layernorm.weight', (h,), NORM_SCALE, 1.0),
        ]
    specs.append(('model.norm.weight', (h,), NORM_SCALE, 1.0))
    if not cfg.tied:
        specs.append(('lm_head.weight', (cfg.vocab, h), MATRIX_SCALE, 0.0))
    return specs


def _mix(z):
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def stream_key(seed: int, tid: int) -> int:
    z = (seed * _GOLDEN + tid * _TENSOR_MUL + 1) & _MASK64
    with np.errstate(over='ignore'):
        return int(_mix(np.array([z], dtype=np.uint64))[0])


def synth_values_numpy(seed: int, tid: int, n: int, scale: float, offset: float,
                       start: int = 0) -> np.ndarray:
    """Pure-numpy restatement of the native filler (slow; for cross-checks)."""
    key = np.uint64(stream_key(seed, tid))
    idx = np.arange(start, start + n, dtype=np.uint64)
    with np.errstate(over='ignore'):
        z = _mix(key + idx * np.uint64(_GOLDEN))
    k = ((z >> np.uint64(40)).astype(np.int64) - (1 << 23)).astype(np.float32)
    step = np.float32(scale) * np.float32(2.0 ** -23)
    return k * step + np.float32(offset)


def _numpy_fill(dst: np.ndarray, seed: int, tid: int, scale: float, offset: float, pool, chunk: int = 1 << 22):
    """:func:`synth_values_numpy` over ``dst`` (flat float32) in chunks on a thread pool
    (numpy's ufuncs release the GIL on large arrays)."""
    def one(start):
        n = min(chunk, dst.size - start)
        dst[start:start + n] = synth_values_numpy(seed, tid, n, scale, offset, start=start)
    list(pool.map(one, range(0, dst.size, chunk)))


def synth_weights(cfg: ModelConfig, seed: int = 0, device: str = 'cpu', backend: str = 'native',
                  threads: int = 1):
    """All weights as float32 torch tensors (HF names).

    ``backend='native'``: on ``device='cuda'`` the CUDA filler writes straight
    into HBM, on the host the multi-threaded native filler runs.
    ``backend='numpy'``: :func:`synth_values_numpy` in chunks on ``threads``
    host threads (no native library involved).  All three are bit-identical.
    """
    import concurrent.futures
    import torch
    out = {}
    pool = concurrent.futures.ThreadPoolExecutor(max_workers=max(1, threads)) if backend == 'numpy' else None
    for tid, (name, shape, scale, offset) in enumerate(tensor_specs(cfg)):
        if backend == 'numpy':
            flat = np.empty(int(np.prod(shape)), dtype=np.float32)
            _numpy_fill(flat, seed, tid, scale, offset, pool)
            t = torch.from_numpy(flat.reshape(shape)).to(device)
        else:
            from . import _native
            t = torch.empty(shape, dtype=torch.float32, device=device)
            _native.synth_fill(t, seed, tid, scale, offset)
        out[name] = t
    if pool is not None:
        pool.shutdown()
    if cfg.tied:
        out['lm_head.weight'] = out['model.embed_tokens.weight']
    return out


def to_bf16(weights):
    """Round-to-nearest-even bf16 copies, as ``model.to(torch.bfloat16)`` does."""
    import torch
    return {k: v.to(torch.bfloat16) for k, v in weights.items()}


# ---------------------------------------------------------------- catalog --

def sid_tokens(cfg: ModelConfig, codes):
    base = cfg.sid_base
    return tuple(base + SID_CODES * level + int(c) for level, c in enumerate(codes))


def catalog_items(wl: Workload):
    """``wl.items`` unique uniform-random SID triples (token ids), in draw order."""
    rng = np.random.Generator(np.random.PCG64(wl.catalog_seed))
    seen, items = set(), []
    while len(items) < wl.items:
        codes = tuple(int(x) for x in rng.integers(0, SID_CODES, size=SID_LEVELS))
        if codes not in seen:
            seen.add(codes)
            items.append(sid_tokens(wl.model, codes))
    return items


def constraint_dict(cfg: ModelConfig, items):
    """The reference's prefix -> allowed-next-tokens dictionary.

    Same construction as ``benchmark_inference.py:87-91``: the root maps to first
    SID tokens, SID prefixes map to their children, a full SID maps to the
    newline and SID+newline maps to EOS.
    """
    root = tuple(cfg.root)
    constraints = collections.defaultdict(set)
    for sid in items:
        ids = list(root) + list(sid) + [cfg.newline, cfg.eos]
        for j in range(3, len(ids)):
            constraints[tuple(ids[:j] if j == 3 else ids[3:j])].add(ids[j])
    return {k: sorted(v) for k, v in constraints.items()}


# ------------------------------------------------------------------ users --

@dataclasses.dataclass(frozen=True)
class User:
    cohort_index: int
    prompt_token_ids: tuple

    @property
    def prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)


def _free_tokens(cfg: ModelConfig):
    banned = {cfg.eos, cfg.newline, *cfg.root}
    lo = min(300, cfg.sid_base // 4)
    return np.array([t for t in range(lo, cfg.sid_base) if t not in banned], dtype=np.int64)


def users(wl: Workload, items=None, count: int | None = None):
    """Seeded prompts: template + filler + history SID triples + root."""
    cfg = wl.model
    items = catalog_items(wl) if items is None else items
    rng = np.random.Generator(np.random.PCG64(wl.prompt_seed))
    free = _free_tokens(cfg)
    template = rng.choice(free, size=wl.template_tokens).tolist()
    out = []
    for u in range(wl.users if count is None else count):
        if wl.prompt_max:
            length = int(rng.integers(wl.prompt_min, wl.prompt_max + 1))
            hmax = min(wl.history_max, (length - wl.template_tokens - 3) // 3)
            hist = int(rng.integers(min(wl.history_min, hmax), hmax + 1))
        else:
            hist = int(rng.integers(wl.history_min, wl.history_max + 1))
            length = wl.template_tokens + 3 * hist + 3
        picks = rng.choice(len(items), size=hist, replace=False)
        filler = rng.choice(free, size=length - wl.template_tokens - 3 * hist - 3).tolist()
        ids = template + filler + [t for p in picks for t in items[int(p)]] + list(cfg.root)
        assert len(ids) == length
        out.append(User(u, tuple(int(x) for x in ids)))
    return out
