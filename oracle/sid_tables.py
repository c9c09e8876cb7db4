"""Numpy restatement of the reference's SID constraint tables and lookup.

Follows ``rapidtinyrec/gpu_constraints.py``:
* grammar check and dense tables: ``GpuSidConstraintTables.__init__`` (:18-67);
* digit index with range check: ``_index`` (:69-73);
* per-step allowed columns: ``lookup`` (:75-87).
The semantic ground truth it must agree with is the released processor's
``prefix_allowed_tokens_fn`` lookup with EOS fallback
(``source/LogitProcessor.py:45-73``), i.e. ``constraints.get(prefix, [eos])``.
"""
from __future__ import annotations

import collections
import math

import numpy as np


class SidTablesOracle:
    def __init__(self, constraints, root_prefix, newline_id, eos_id):
        root_prefix = tuple(root_prefix)
        assert len(root_prefix) == 3
        sids = sorted(k for k in constraints if len(k) == 3 and k != root_prefix)
        assert sids and all(len(s) == 3 for s in sids)
        canonical = collections.defaultdict(set)
        for sid in sids:                                   # gpu_constraints.py:24-29
            canonical[root_prefix].add(sid[0])
            canonical[sid[:1]].add(sid[1])
            canonical[sid[:2]].add(sid[2])
            canonical[sid].add(newline_id)
            canonical[sid + (newline_id,)].add(eos_id)
        assert dict(canonical) == {k: set(v) for k, v in constraints.items()}, 'Unexpected SID grammar'
        self.offsets = [min(s[i] for s in sids) for i in range(3)]          # :31
        self.sizes = [max(s[i] for s in sids) - self.offsets[i] + 1 for i in range(3)]  # :32
        assert math.prod(self.sizes) <= 100_000_000
        self.root = root_prefix
        self.newline, self.eos = newline_id, eos_id
        self.first_tokens = np.array(sorted(canonical[root_prefix]), dtype=np.int64)
        self.tables = {}
        for n in (1, 2):                                    # :44-55
            width = max(len(v) for k, v in canonical.items() if len(k) == n)
            table = np.full((math.prod(self.sizes[:n]), width), eos_id, dtype=np.int64)
            for key, allowed in canonical.items():
                if len(key) != n:
                    continue
                index = sum((key[j] - self.offsets[j]) * math.prod(self.sizes[j + 1:n]) for j in range(n))
                tokens = sorted(allowed)
                table[index] = tokens + [tokens[0]] * (width - len(tokens))
            self.tables[n] = table
        valid = np.zeros(math.prod(self.sizes), dtype=bool)  # :56-60
        for sid in sids:
            valid[sum((sid[j] - self.offsets[j]) * math.prod(self.sizes[j + 1:]) for j in range(3))] = True
        self.valid = valid

    def _index(self, tokens, n):                            # :69-73
        digits = tokens - np.array(self.offsets[:n], dtype=np.int64)
        in_range = ((digits >= 0) & (digits < np.array(self.sizes[:n]))).all(axis=-1)
        strides = np.array([math.prod(self.sizes[j + 1:n]) for j in range(n)], dtype=np.int64)
        index = (digits * strides).sum(axis=-1)
        return np.clip(index, 0, math.prod(self.sizes[:n]) - 1), in_range

    def lookup(self, step, input_ids):
        """Allowed-column rows for ``input_ids [rows, cur_len]`` at ``step`` (:75-87)."""
        input_ids = np.asarray(input_ids, dtype=np.int64)
        rows = input_ids.shape[0]
        if step in (1, 2):
            index, in_range = self._index(input_ids[:, -step:], step)
            return np.where(in_range[:, None], self.tables[step][index], self.eos)
        if step in (0, 3):
            suffix = input_ids[:, -3:]
            index, in_range = self._index(suffix, 3)
            terminal = np.where(in_range & self.valid[index], self.newline, self.eos)
            is_root = (suffix == np.array(self.root)).all(axis=-1)
            width = len(self.first_tokens)
            return np.where(is_root[:, None], self.first_tokens[None, :],
                            np.broadcast_to(terminal[:, None], (rows, width)))
        return np.full((rows, 1), self.eos, dtype=np.int64)


def semantic_allowed(constraints, eos_id, step, prefix_ids):
    """Released-processor semantics: ``constraints.get(key, [])`` or EOS fallback.

    ``source/LogitProcessor.py:52-68``: the key is the last ``prefix_index`` (3)
    tokens at step 0 and the last ``count`` tokens afterwards.
    """
    key = tuple(int(x) for x in (prefix_ids[-3:] if step == 0 else prefix_ids[-step:]))
    allowed = constraints.get(key, [])
    return sorted(set(allowed)) if allowed else [eos_id]
