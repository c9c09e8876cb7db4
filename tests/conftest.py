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


def fake_tokenizer(codes=8):
    """A word-level tokenizer for the release layout: '### ', 'Response', ':\\n' (the
    response root, like Qwen's three tokens), the newline,
    SID pieces <a_i>/<b_i>/<c_i> and a few words, each one token."""
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {'<unk>': 0, '<eos>': 1, '### ': 2, 'Response': 3, ':\n': 4, '\n': 5}
    for level in 'abc':
        for code in range(codes):
            vocab[f'<{level}_{code}>'] = len(vocab)
    for w in ('hello', 'world', 'office', 'paper', 'pen'):
        vocab[w] = len(vocab)
    tk = Tokenizer(models.WordLevel(vocab, unk_token='<unk>'))
    tk.pre_tokenizer = pre_tokenizers.Split(Regex(r'<[abc]_\d+>|### |Response|:\n|\n|\w+'), behavior='isolated')
    return PreTrainedTokenizerFast(tokenizer_object=tk, eos_token='<eos>', unk_token='<unk>'), vocab


def write_fake_release(root, sids, n_users=3, hidden=64, heads=4, kv_heads=2, intermediate=96, layers=2,
                       vocab_size=64, codes=8, seed=0):
    """Checkpoint + tokenizer + catalog + reference manifest in the reference's release layout."""
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from rapidtinyrec_b200 import release
    tok, vocab = fake_tokenizer(codes)
    ckpt = root / release.CHECKPOINT
    tok.save_pretrained(ckpt)
    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=vocab_size, hidden_size=hidden, intermediate_size=intermediate,
                      num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                      rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=512)
    Qwen2ForCausalLM(cfg).save_pretrained(ckpt)
    cat = root / release.CATALOG
    cat.parent.mkdir(parents=True)
    cat.write_text(''.join(f'{s}\tsome title {i}\n' for i, s in enumerate(sids)))
    rootids = [vocab['### '], vocab['Response'], vocab[':\n']]
    words = [vocab[w] for w in ('hello', 'world', 'office', 'paper', 'pen')]
    rng = np.random.default_rng(seed)
    users = []
    for i in range(n_users):
        body = [int(x) for x in rng.choice(words, size=4 + 2 * i)]
        hist = [vocab[t] for s in sids[i:i + 2] for t in ('<' + x for x in s.split('<')[1:])]
        ids = body + hist + rootids
        users.append({'cohort_index': i, 'prompt_tokens': len(ids), 'user_id': f'u{i}', 'prompt_token_ids': ids,
                      'target_sid': sids[(i + 2) % len(sids)]})  # the held-out next item
    res = root / 'reference_results'
    res.mkdir()
    (res / 'manifest.json').write_text(json.dumps({'users': users}))
    return res, vocab
