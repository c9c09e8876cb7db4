"""Semantic-ID constraint tables and processor: the reference's plugin API, native.

``GpuSidConstraintTables`` keeps the reference's constructor, grammar check and
error text (``rapidtinyrec/gpu_constraints.py:17-67``) and builds the same
dense tables on the host; ``upload`` hands them to a native session, whose
kernels do every lookup on device.  ``GpuSidConstrainedLogitsProcessor`` is the
Hugging Face ``LogitsProcessor`` drop-in (``gpu_constraints.py:90-101``)
running the native normalisation + mask kernel.
"""
from __future__ import annotations

import collections
import ctypes
import math

import numpy as np

from . import _native


class GpuSidConstraintTables:
    def __init__(self, constraints, root_prefix, newline_id, eos_id, device='cuda'):
        root_prefix = tuple(root_prefix)
        assert len(root_prefix) == 3
        sids = sorted(key for key in constraints if len(key) == 3 and key != root_prefix)
        assert sids and all(len(sid) == 3 for sid in sids)
        canonical = collections.defaultdict(set)
        for sid in sids:
            canonical[root_prefix].add(sid[0])
            canonical[sid[:1]].add(sid[1])
            canonical[sid[:2]].add(sid[2])
            canonical[sid].add(newline_id)
            canonical[sid + (newline_id,)].add(eos_id)
        assert dict(canonical) == {k: set(v) for k, v in constraints.items()}, 'Unexpected SID grammar'
        offsets = [min(sid[i] for sid in sids) for i in range(3)]
        sizes = [max(sid[i] for sid in sids) - offsets[i] + 1 for i in range(3)]
        assert math.prod(sizes) <= 100_000_000, 'Dense SID-validity table too large for this implementation'
        self.device = device
        self.offsets, self.sizes = offsets, sizes
        self.root_prefix = root_prefix
        self.newline, self.eos = int(newline_id), int(eos_id)
        self.first_tokens = np.array(sorted(canonical[root_prefix]), dtype=np.int32)
        self.tables = {}
        for n in (1, 2):
            width = max(len(v) for k, v in canonical.items() if len(k) == n)
            table = np.full((math.prod(sizes[:n]), width), eos_id, dtype=np.int32)
            for key, allowed in canonical.items():
                if len(key) != n:
                    continue
                index = sum((key[j] - offsets[j]) * math.prod(sizes[j + 1:n]) for j in range(n))
                tokens = sorted(allowed)
                table[index] = tokens + [tokens[0]] * (width - len(tokens))
            self.tables[n] = table
        valid = np.zeros(math.prod(sizes), dtype=np.uint8)
        for sid in sids:
            valid[sum((sid[j] - offsets[j]) * math.prod(sizes[j + 1:]) for j in range(3))] = 1
        self.valid_sids = valid
        self.metadata = {'unique_sids': len(sids), 'sid_offsets': offsets, 'sid_range_sizes': sizes,
                         'device_table_bytes': int(sum(t.nbytes for t in self.tables.values()) + valid.nbytes
                                                   + self.first_tokens.nbytes),
                         'table_shapes': {str(n): list(t.shape) for n, t in self.tables.items()},
                         'unknown_prefix_behavior': 'EOS fallback on device',
                         'runtime_cpu_token_transfers': 0}

    def host_arrays(self):
        """Every table as a host array (for the runner's unchanged-input audit)."""
        return {'offsets': np.array(self.offsets, np.int64), 'sizes': np.array(self.sizes, np.int64),
                'tables.1': self.tables[1], 'tables.2': self.tables[2], 'valid_sids': self.valid_sids,
                'first_tokens': self.first_tokens, 'root_prefix': np.array(self.root_prefix, np.int64)}

    def as_c(self):
        """The ``rtr_constraint_tables`` struct (host pointers kept alive by ``self``)."""
        self._keep = [np.ascontiguousarray(self.tables[1]), np.ascontiguousarray(self.tables[2]),
                      np.ascontiguousarray(self.valid_sids), np.ascontiguousarray(self.first_tokens)]
        t1, t2, valid, first = self._keep
        i32p = ctypes.POINTER(ctypes.c_int32)
        return _native.ConstraintTablesC(
            offsets=(ctypes.c_int32 * 3)(*self.offsets), sizes=(ctypes.c_int32 * 3)(*self.sizes),
            table1=t1.ctypes.data_as(i32p), width1=t1.shape[1],
            table2=t2.ctypes.data_as(i32p), width2=t2.shape[1],
            valid=valid.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
            root=(ctypes.c_int32 * 3)(*self.root_prefix),
            first_tokens=first.ctypes.data_as(i32p), n_first=len(first),
            newline=self.newline, eos=self.eos)


class GpuSidConstrainedLogitsProcessor:
    """``LogitsProcessor`` drop-in: ``scores -> log_softmax(scores) + mask``.

    The step counter advances per call, as in the reference (``count``).
    """

    def __init__(self, tables, session):
        self.tables = tables
        self.session = session
        self.count = 0

    def __call__(self, input_ids, scores):
        import torch
        if not (scores.is_cuda and input_ids.is_cuda):
            raise ValueError('native processor needs CUDA tensors')
        ids = input_ids.to(torch.int64).contiguous()
        src = scores.to(torch.float32).contiguous()
        out = torch.empty_like(src)
        self.session.constraint_process(self.count, ids, src, out)
        self.count += 1
        return out
