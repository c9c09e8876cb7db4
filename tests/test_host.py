"""Host-side logic and the C ABI surface (no GPU needed)."""
import ctypes
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, GOLDEN
from oracle.sid_tables import SidTablesOracle
from rapidtinyrec_b200 import _native, configs, workload
from rapidtinyrec_b200.constraints import GpuSidConstraintTables
from rapidtinyrec_b200.engine import rope_table, weight_order
from tests.golden.make_golden import grammar_444, catalog_5x5x4


def test_header_declares_exactly_the_exports():
    header = (ROOT / 'include' / 'rtr_b200.h').read_text()
    declared = set(re.findall(r'^\s*(?:int|const char\*)\s+(rtr_\w+)\(', header, re.M))
    assert declared == set(_native.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    lib = _native.load()
    for name in _native.EXPORTS:
        assert hasattr(lib, name), name


def test_create_rejects_bad_config_without_gpu_work():
    lib = _native.load()
    h = ctypes.c_void_p()
    bad = _native.ModelConfigC(layers=1, hidden=64, heads=3, kv_heads=2, head_dim=64, intermediate=64,
                               vocab=512, tied_embeddings=1, rms_eps=1e-6, rope_theta=1e4,
                               dtype=0, max_prefix=16, num_beams=50)
    assert lib.rtr_session_create(ctypes.byref(bad), 0, ctypes.byref(h)) == _native.RTR_ERR_ARG
    assert b'multiple' in lib.rtr_last_error(None)
    bad.heads, bad.head_dim = 4, 32
    assert lib.rtr_session_create(ctypes.byref(bad), 0, ctypes.byref(h)) == _native.RTR_ERR_ARG
    bad.head_dim, bad.num_beams = 64, 65
    assert lib.rtr_session_create(ctypes.byref(bad), 0, ctypes.byref(h)) == _native.RTR_ERR_ARG


@pytest.mark.parametrize('seed,tid,scale,offset', [(0, 0, 0.0346, 0.0), (0, 17, 0.1, 1.0), (9, 3, 0.5, -0.25)])
def test_native_host_filler_matches_numpy(seed, tid, scale, offset):
    t = torch.empty(70001)
    _native.synth_fill(t, seed, tid, scale, offset)
    assert np.array_equal(t.numpy(), workload.synth_values_numpy(seed, tid, 70001, scale, offset))


def test_synth_weights_backends_agree():
    cfg = configs.ModelConfig('t', layers=1, hidden=32, heads=2, kv_heads=1, head_dim=16, intermediate=48,
                              vocab=800, tied=False, dtype='fp32', eos=5, root=(1, 2, 3))
    a = workload.synth_weights(cfg, backend='numpy')
    b = workload.synth_weights(cfg, backend='native')
    assert set(a) == set(b) == set(weight_order(cfg))
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert abs(float(a['model.layers.0.mlp.up_proj.weight'].std()) - 0.02) < 2e-3
    assert float(a['model.norm.weight'].min()) >= 0.9


@pytest.mark.parametrize('name', ['test_catalog', 'grammar_444', 'tiny'])
def test_product_tables_equal_oracle_tables(name, tiny):
    if name == 'test_catalog':
        cons, root, nl, eos = catalog_5x5x4(), (1, 2, 3), 510, 511
    elif name == 'grammar_444':
        cons, root, nl, eos = grammar_444(), (1, 2, 3), 4, 5
    else:
        cfg = tiny['cfg']
        cons, root, nl, eos = tiny['constraints'], cfg.root, cfg.newline, cfg.eos
    prod = GpuSidConstraintTables(cons, root, nl, eos)
    ref = SidTablesOracle(cons, root, nl, eos)
    assert prod.offsets == ref.offsets and prod.sizes == ref.sizes
    for n in (1, 2):
        assert np.array_equal(prod.tables[n], ref.tables[n])
    assert np.array_equal(prod.valid_sids.astype(bool), ref.valid)
    assert np.array_equal(prod.first_tokens, ref.first_tokens)
    c = prod.as_c()
    assert c.width1 == prod.tables[1].shape[1] and c.n_first == len(prod.first_tokens)


def test_product_tables_reject_bad_grammar():
    cons = dict(catalog_5x5x4())
    cons[(40, 70, 100)] = [510, 7]
    with pytest.raises(AssertionError, match='Unexpected SID grammar'):
        GpuSidConstraintTables(cons, (1, 2, 3), 510, 511)


def test_workload_is_deterministic_and_well_formed():
    wl = configs.workload('qwen1.5b-fp32')
    items = workload.catalog_items(wl)
    assert len(items) == len(set(items)) == 3500
    cfg = wl.model
    assert all(cfg.sid_base <= t < cfg.vocab for it in items for t in it)
    us = workload.users(wl, items, count=40)
    assert us == workload.users(wl, items, count=40)
    for u in us:
        assert 150 <= u.prompt_tokens <= 350
        assert tuple(u.prompt_token_ids[-3:]) == cfg.root
        assert all(0 <= t < cfg.vocab for t in u.prompt_token_ids)
    cons = workload.constraint_dict(cfg, items)
    tables = GpuSidConstraintTables(cons, cfg.root, cfg.newline, cfg.eos)
    assert tables.sizes == [256, 256, 256] or max(tables.sizes) <= 256
    assert len(tables.first_tokens) >= 50


def test_rope_table_matches_oracle_formula():
    from oracle.qwen2_cpu import rope_table as oracle_rope
    for d, theta in ((128, 1e6), (64, 1e6)):
        c1, s1 = rope_table(d, theta, 300)
        c2, s2 = oracle_rope(d, theta, 300)
        assert np.array_equal(c1, c2.numpy()) and np.array_equal(s1, s2.numpy())


def test_weight_bytes_per_step_primary():
    cfg = configs.workload('qwen1.5b-fp32').model
    assert cfg.weight_bytes_per_step() == 6_179_575_808
    assert cfg.kv_bytes_per_token() == 57_344
