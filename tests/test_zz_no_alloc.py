"""The allocation-free processor entry point, through the C ABI.

rtr_constraint_process_static serves callers that may not allocate device
memory per call (a plugin under a host framework's allocator that has reserved
the GPU's memory): it keeps its reduction scratch in a static device array of
the library.  Its scores must match
rtr_constraint_process - the entry point that uses session-allocated scratch -
within the processor tolerance, call after call, since every call reuses the
same array.  The file sorts last so a failure here comes after every other
test has run.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

PROCESSOR_TOL = 4e-6  # same bound as the processor parity test


def _engine(tiny):
    from rapidtinyrec_b200 import configs
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine
    c = tiny['cfg']
    cfg = configs.ModelConfig('tables', layers=1, hidden=64, heads=1, kv_heads=1, head_dim=64, intermediate=64,
                              vocab=c.vocab, tied=True, dtype='fp32', newline=c.newline, eos=c.eos, root=c.root)
    tables = GpuSidConstraintTables(tiny['constraints'], c.root, c.newline, c.eos)
    return BeamEngine(cfg, None, tables, max_prefix=16)


def _call(lib, eng, name, step, ids, scores, out):
    fn = getattr(lib, name)
    code = fn(eng.handle, step, ctypes.c_void_p(ids.data_ptr()), ids.shape[0], ids.shape[1],
              ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(out.data_ptr()))
    return code


def test_static_scratch_processor_matches_session_scratch(tiny):
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required')
    from rapidtinyrec_b200 import _native
    lib = _native.load()
    eng = _engine(tiny)
    dev = torch.device('cuda:0')
    vocab = eng.cfg.vocab
    z = np.load(GOLDEN / 'processor_tiny.npz')
    gen = torch.Generator().manual_seed(7)
    for call, step in enumerate((0, 1)):  # two calls in a row on the shared array
        scores = torch.randn((50, vocab), generator=gen).to(dev)
        ids = torch.from_numpy(z[f'input_{step}'].astype(np.int64)).to(dev)
        want = torch.empty_like(scores)
        got = torch.full_like(scores, float('nan'))
        torch.cuda.synchronize()
        assert _call(lib, eng, 'rtr_constraint_process', step, ids, scores, want) == _native.RTR_OK
        assert _call(lib, eng, 'rtr_constraint_process_static', step, ids, scores, got) == _native.RTR_OK, \
            lib.rtr_last_error(eng.handle)
        finite_w, finite_g = torch.isfinite(want), torch.isfinite(got)
        assert torch.equal(finite_w, finite_g), call
        assert int(finite_g.sum()) > 0
        assert float((got[finite_g] - want[finite_w]).abs().max()) <= PROCESSOR_TOL, call
        assert torch.equal(got[~finite_g], want[~finite_w])  # -inf outside the allowed columns


def test_static_scratch_processor_allocates_nothing(tiny):
    """Free device memory is the same before and after repeated calls."""
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required')
    from rapidtinyrec_b200 import _native
    lib = _native.load()
    eng = _engine(tiny)
    dev = torch.device('cuda:0')
    z = np.load(GOLDEN / 'processor_tiny.npz')
    scores = torch.randn((50, eng.cfg.vocab), generator=torch.Generator().manual_seed(3)).to(dev)
    ids = torch.from_numpy(z['input_0'].astype(np.int64)).to(dev)
    out = torch.empty_like(scores)
    assert _call(lib, eng, 'rtr_constraint_process_static', 0, ids, scores, out) == _native.RTR_OK  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(5):
        assert _call(lib, eng, 'rtr_constraint_process_static', 0, ids, scores, out) == _native.RTR_OK
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, (free0, free1)


def test_static_scratch_processor_rejects_rows_beyond_its_array(tiny):
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required')
    from rapidtinyrec_b200 import _native
    lib = _native.load()
    eng = _engine(tiny)
    dev = torch.device('cuda:0')
    scores = torch.zeros((257, eng.cfg.vocab), device=dev)
    out = torch.empty_like(scores)
    ids = torch.zeros((257, 3), dtype=torch.int64, device=dev)
    assert _call(lib, eng, 'rtr_constraint_process_static', 0, ids, scores, out) == _native.RTR_ERR_ARG
    assert b'256 rows' in lib.rtr_last_error(eng.handle)
