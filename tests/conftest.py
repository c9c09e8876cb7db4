import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / 'tests' / 'golden'
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200) and the built native library')


def load_generate_fixture(name):
    meta = json.loads((GOLDEN / f'generate_{name}.json').read_text())
    arrays = np.load(GOLDEN / f'generate_{name}.npz')
    return meta, arrays


def fixture_weights(arrays):
    import torch
    return {k[2:]: torch.from_numpy(arrays[k]) for k in arrays.files if k.startswith('w:')}


@pytest.fixture(scope='session')
def tiny():
    """Tiny workload: config, catalog, constraints, users, weights (numpy generator)."""
    from rapidtinyrec_b200 import configs, workload
    wl = configs.workload('tiny')
    items = workload.catalog_items(wl)
    return {
        'wl': wl, 'cfg': wl.model, 'items': items,
        'constraints': workload.constraint_dict(wl.model, items),
        'users': workload.users(wl, items),
        'weights': workload.synth_weights(wl.model, seed=wl.weight_seed, backend='numpy'),
    }
