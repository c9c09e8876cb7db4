"""Model shapes and synthetic request workloads for the semantic-ID beam path.

Every workload is a Qwen2-architecture decoder (RMSNorm, GQA attention with
q/k/v bias, RoPE, SwiGLU MLP) whose vocabulary ends in 768 semantic-ID (SID)
tokens: three levels of 256 codes each, level ``l`` code ``c`` being token
``sid_base + 256*l + c``.  The model shapes follow the MiniOneRec release the
reference benchmarks (Qwen2 1.5B, ``benchmark_inference.py:93-98``); the
request shape follows ``EvalSidDataset`` (instruction, history SIDs, then the
three-token ``### Response:\\n`` root, ``source/data.py:604-658``).

The real release (checkpoint, tokenizer, Amazon catalog) is not available, so
weights, catalogs and prompts are seeded synthetic stand-ins with the same
shapes: weights seed 0, catalog seed 1, prompts seed 2.
"""
from __future__ import annotations

import dataclasses

SID_LEVELS = 3
SID_CODES = 256
NUM_BEAMS = 50
# Prefill output + four decode forwards: three SID tokens, newline, EOS
# (``benchmark_inference.py:147`` asserts exactly five forward calls).
NUM_STEPS = 5


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    tied: bool
    dtype: str            # 'fp32' or 'bf16': weights, activations and KV
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    newline: int = 198
    eos: int = 151643
    root: tuple = (14374, 5949, 510)

    @property
    def sid_base(self) -> int:
        return self.vocab - SID_LEVELS * SID_CODES

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def layer_params(self) -> int:
        h, i = self.hidden, self.intermediate
        return (h * self.qkv_dim + self.qkv_dim + h * self.q_dim + 3 * h * i + 2 * h)

    def weight_bytes_per_step(self) -> int:
        """Algorithmic weight bytes one decode step streams (layers + LM head + final norm)."""
        b = 4 if self.dtype == 'fp32' else 2
        return b * (self.layers * self.layer_params() + self.vocab * self.hidden + self.hidden)

    def kv_bytes_per_token(self) -> int:
        b = 4 if self.dtype == 'fp32' else 2
        return b * 2 * self.kv_dim * self.layers

    def with_dtype(self, dtype: str) -> 'ModelConfig':
        return dataclasses.replace(self, dtype=dtype)


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    model: ModelConfig
    items: int                 # catalog size (unique SID triples)
    users: int
    prompt_min: int
    prompt_max: int
    history_min: int
    history_max: int
    template_tokens: int = 40  # fixed instruction template length
    weight_seed: int = 0
    catalog_seed: int = 1
    prompt_seed: int = 2


TINY = ModelConfig('tiny', layers=4, hidden=256, heads=4, kv_heads=2, head_dim=64,
                   intermediate=688, vocab=8192, tied=True, dtype='fp32',
                   eos=7423, root=(17, 19, 23))
QWEN_1_5B = ModelConfig('qwen2.5-1.5b', layers=28, hidden=1536, heads=12, kv_heads=2,
                        head_dim=128, intermediate=8960, vocab=151936 + 768, tied=True,
                        dtype='fp32')
QWEN_0_5B = ModelConfig('qwen2.5-0.5b', layers=24, hidden=896, heads=14, kv_heads=2,
                        head_dim=64, intermediate=4864, vocab=151936 + 768, tied=True,
                        dtype='fp32')
QWEN_7B = ModelConfig('qwen2.5-7b', layers=28, hidden=3584, heads=28, kv_heads=4,
                      head_dim=128, intermediate=18944, vocab=152064 + 768, tied=False,
                      dtype='bf16')

WORKLOADS = {
    # Tiny: 40-token instruction + 10-20 history items x 3 SID tokens + root.
    'tiny': Workload('tiny', TINY, items=2000, users=8, prompt_min=0, prompt_max=0,
                     history_min=10, history_max=20),
    # Primary: 1.5B FP32, 500 users, prompts of 150-350 tokens, 10-30 history items.
    'qwen1.5b-fp32': Workload('qwen1.5b-fp32', QWEN_1_5B, items=3500, users=500,
                              prompt_min=150, prompt_max=350, history_min=10, history_max=30),
    'qwen1.5b-bf16': Workload('qwen1.5b-bf16', QWEN_1_5B.with_dtype('bf16'), items=3500,
                              users=500, prompt_min=150, prompt_max=350,
                              history_min=10, history_max=30),
    'qwen0.5b-fp32': Workload('qwen0.5b-fp32', QWEN_0_5B, items=10000, users=8000,
                              prompt_min=100, prompt_max=300, history_min=10, history_max=30),
    'qwen7b-bf16': Workload('qwen7b-bf16', QWEN_7B, items=50000, users=2000,
                            prompt_min=600, prompt_max=1024, history_min=40, history_max=100),
}


def workload(name: str) -> Workload:
    try:
        return WORKLOADS[name]
    except KeyError:
        raise ValueError(f'Unknown workload {name!r}; choose from {sorted(WORKLOADS)}') from None
