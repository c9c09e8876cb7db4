"""Host side of the native beam-search engine.

``BeamEngine`` is the B200 replacement for what ``benchmark_inference.run``
assembles around Hugging Face ``generate`` (``rapidtinyrec/benchmark_inference.py:93-148``):
model + ``PrefillPrefix`` + ``PrefixArena`` + ``PrefixReplayPool`` +
``ReorderSuffix`` + ``GpuSidConstrainedLogitsProcessor``.  One engine is one
model replica on one GPU serving sequential requests; every request returns
the reference's per-user record (``benchmark_inference.py:150-154``).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native
from .configs import NUM_BEAMS, NUM_STEPS, ModelConfig


def rope_table(head_dim: int, theta: float, n_positions: int, dtype=None):
    """cos/sin ``[n_positions, head_dim/2]`` with the Qwen2 rotary formula.

    Same float32 torch ops as ``Qwen2RotaryEmbedding`` (transformers
    modeling_qwen2.py:89-113), so the table is bit-identical to the one the
    reference builds on the host.  ``dtype='bf16'`` reproduces a model cast with
    ``.to(torch.bfloat16)``, which also rounds the ``inv_freq`` buffer.
    """
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    if dtype == 'bf16':
        inv = inv.to(torch.bfloat16).float()
    pos = torch.arange(n_positions)[None, None, :].float()
    freqs = (inv[None, :, None].float() @ pos).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    # cos/sin in blocks below torch's parallel grain (32,768 elements) so every
    # element takes the vectorised path, as a single-threaded HF call does; a
    # thread split of the whole table could leave scalar tails with other bits.
    rows = max(1, 16384 // head_dim)
    cos = torch.cat([emb[:, i:i + rows].cos() for i in range(0, n_positions, rows)], dim=1)
    sin = torch.cat([emb[:, i:i + rows].sin() for i in range(0, n_positions, rows)], dim=1)
    return (cos[0, :, :head_dim // 2].contiguous().numpy(),
            sin[0, :, :head_dim // 2].contiguous().numpy())


def weight_order(cfg: ModelConfig):
    """Tensor names in the order ``rtr_load_weights`` expects."""
    names = ['model.embed_tokens.weight']
    for n in range(cfg.layers):
        p = f'model.layers.{n}.'
        names += [p + 'self_attn.q_proj.weight', p + 'self_attn.q_proj.bias',
                  p + 'self_attn.k_proj.weight', p + 'self_attn.k_proj.bias',
                  p + 'self_attn.v_proj.weight', p + 'self_attn.v_proj.bias',
                  p + 'self_attn.o_proj.weight', p + 'mlp.gate_proj.weight', p + 'mlp.up_proj.weight',
                  p + 'mlp.down_proj.weight', p + 'input_layernorm.weight',
                  p + 'post_attention_layernorm.weight']
    names.append('model.norm.weight')
    if not cfg.tied:
        names.append('lm_head.weight')
    return names


class BeamEngine:
    def __init__(self, cfg: ModelConfig, weights, tables, max_prefix: int, device: int = 0,
                 num_beams: int = NUM_BEAMS, max_users: int = 1):
        import torch
        self.lib = _native.load()
        self.cfg = cfg
        self.beams = num_beams
        self.device = device
        self.max_prefix = max_prefix
        self.max_users = max_users
        c = _native.ModelConfigC(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads,
                                 head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab,
                                 tied_embeddings=int(cfg.tied), rms_eps=cfg.rms_eps, rope_theta=cfg.rope_theta,
                                 dtype=_native.RTR_DTYPE_F32 if cfg.dtype == 'fp32' else _native.RTR_DTYPE_BF16,
                                 max_prefix=max_prefix, num_beams=num_beams)
        handle = ctypes.c_void_p()
        _native.check(self.lib.rtr_session_create_batched(ctypes.byref(c), device, max_users, ctypes.byref(handle)))
        self.handle = handle
        try:
            if weights is not None:
                self._load_weights(weights)
            cos, sin = rope_table(cfg.head_dim, cfg.rope_theta, max_prefix + 8, cfg.dtype)
            self._check(self.lib.rtr_load_rope(self.handle, cos.ctypes.data, sin.ctypes.data, cos.shape[0]))
            self.tables = tables
            self._check(self.lib.rtr_load_constraints(self.handle, ctypes.byref(tables.as_c())))
        except Exception:
            self.close()
            raise
        self._tok = np.zeros(num_beams * NUM_STEPS, dtype=np.int32)
        self._par = np.zeros(num_beams * NUM_STEPS, dtype=np.int32)
        self._seq = np.zeros(num_beams, dtype=np.float32)
        self._trans = np.zeros(num_beams * NUM_STEPS, dtype=np.float32)
        i32p, f32p = ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float)
        self._result = _native.ResultC(self._tok.ctypes.data_as(i32p), self._par.ctypes.data_as(i32p),
                                       self._seq.ctypes.data_as(f32p), self._trans.ctypes.data_as(f32p))
        # one result record per user of a batch
        self._btok = np.zeros((max_users, num_beams * NUM_STEPS), dtype=np.int32)
        self._bpar = np.zeros_like(self._btok)
        self._bseq = np.zeros((max_users, num_beams), dtype=np.float32)
        self._btrans = np.zeros((max_users, num_beams * NUM_STEPS), dtype=np.float32)
        self._bresults = (_native.ResultC * max_users)(*[
            _native.ResultC(self._btok[u].ctypes.data_as(i32p), self._bpar[u].ctypes.data_as(i32p),
                            self._bseq[u].ctypes.data_as(f32p), self._btrans[u].ctypes.data_as(f32p))
            for u in range(max_users)])
        self._batch_n = 0
        del torch

    # ------------------------------------------------------------ plumbing
    def _check(self, code):
        return _native.check(code, self.handle)

    def _load_weights(self, weights):
        import torch
        names = weight_order(self.cfg)
        tensors = []
        on_device = None
        for n in names:
            t = weights[n]
            if t.dtype != torch.float32:
                t = t.float()
            t = t.contiguous()
            dev = bool(t.is_cuda)
            if on_device is None:
                on_device = dev
            elif on_device != dev:
                t = t.cuda(self.device) if on_device else t.cpu()
            tensors.append(t)
        ptrs = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
        if on_device:
            torch.cuda.synchronize(self.device)
        self._check(self.lib.rtr_load_weights(self.handle, ptrs, len(tensors), _native.RTR_DTYPE_F32,
                                              int(bool(on_device))))

    def close(self):
        if getattr(self, 'handle', None) and self.handle.value:
            self.lib.rtr_session_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _record(self):
        b = self.beams
        return {'beam_indices': self._par.reshape(b, NUM_STEPS).tolist(),
                'score_dtypes': ['torch.float32'] * NUM_STEPS,
                'token_ids': self._tok.reshape(b, NUM_STEPS).tolist(),
                'sequence_logp': self._seq.tolist(),
                'transition_logp': self._trans.reshape(b, NUM_STEPS).tolist()}

    def _batch_records(self, n):
        b = self.beams
        return [{'beam_indices': self._bpar[u].reshape(b, NUM_STEPS).tolist(),
                 'score_dtypes': ['torch.float32'] * NUM_STEPS,
                 'token_ids': self._btok[u].reshape(b, NUM_STEPS).tolist(),
                 'sequence_logp': self._bseq[u].tolist(),
                 'transition_logp': self._btrans[u].reshape(b, NUM_STEPS).tolist()} for u in range(n)]

    @staticmethod
    def _ids(prompt_ids):
        ids = np.ascontiguousarray(np.asarray(prompt_ids, dtype=np.int32).reshape(-1))
        return ids

    # ------------------------------------------------------------- requests
    def generate(self, prompt_ids):
        """One request end to end (prefill + one decode graph); the reference's record."""
        ids = self._ids(prompt_ids)
        self._check(self.lib.rtr_generate(self.handle, ids.ctypes.data, len(ids), ctypes.byref(self._result)))
        return self._record()

    def generate_batch(self, prompts):
        """Several users in one request (session built with ``max_users``): each
        user's prefill, then their decode steps together; one record per user."""
        ids = [self._ids(p) for p in prompts]
        n = len(ids)
        ptrs = (ctypes.c_void_p * n)(*[a.ctypes.data for a in ids])
        lens = (ctypes.c_int32 * n)(*[len(a) for a in ids])
        self._check(self.lib.rtr_generate_batch(self.handle, ptrs, lens, n, self._bresults))
        return self._batch_records(n)

    def launch_batch_device(self, ids_dev, lengths):
        """Enqueue one batched request whose prompts already sit in device memory."""
        n = len(ids_dev)
        ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in ids_dev])
        lens = (ctypes.c_int32 * n)(*lengths)
        self._check(self.lib.rtr_launch_batch(self.handle, ptrs, lens, n, 1))
        self._batch_n = n

    def wait_batch(self):
        self._check(self.lib.rtr_wait_batch(self.handle, self._bresults))
        return self._batch_records(self._batch_n)

    def generate_raw(self, ids: np.ndarray):
        """``generate`` without building the Python record (for timing loops)."""
        self._check(self.lib.rtr_generate(self.handle, ids.ctypes.data, len(ids), ctypes.byref(self._result)))

    def prefill(self, prompt_ids):
        ids = self._ids(prompt_ids)
        self._check(self.lib.rtr_prefill(self.handle, ids.ctypes.data, len(ids), 0))

    def decode_step(self, t):
        self._check(self.lib.rtr_decode_step(self.handle, t))

    def read_results(self):
        self._check(self.lib.rtr_read_results(self.handle, ctypes.byref(self._result)))
        return self._record()

    def step_scores(self, t):
        """``GenerateBeamOutput.scores[t]``: dense ``[beams, V]`` float32 CUDA tensor."""
        import torch
        out = torch.empty((self.beams, self.cfg.vocab), dtype=torch.float32, device=f'cuda:{self.device}')
        self._check(self.lib.rtr_step_scores(self.handle, t, ctypes.c_void_p(out.data_ptr())))
        return out

    # ------------------------------------------------- plugin entry points
    def lookup_width(self, step):
        w = ctypes.c_int32()
        self._check(self.lib.rtr_lookup_width(self.handle, step, ctypes.byref(w)))
        return w.value

    def constraint_lookup(self, step, input_ids):
        import torch
        ids = input_ids.to(device=f'cuda:{self.device}', dtype=torch.int64).contiguous()
        out = torch.empty((ids.shape[0], self.lookup_width(step)), dtype=torch.int32, device=ids.device)
        torch.cuda.synchronize(self.device)
        self._check(self.lib.rtr_constraint_lookup(self.handle, step, ctypes.c_void_p(ids.data_ptr()),
                                                   ids.shape[0], ids.shape[1], ctypes.c_void_p(out.data_ptr())))
        return out

    def constraint_process(self, step, input_ids, scores, out):
        import torch
        torch.cuda.synchronize(self.device)
        self._check(self.lib.rtr_constraint_process(self.handle, step, ctypes.c_void_p(input_ids.data_ptr()),
                                                    input_ids.shape[0], input_ids.shape[1],
                                                    ctypes.c_void_p(scores.data_ptr()),
                                                    ctypes.c_void_p(out.data_ptr())))
        return out

    # ------------------------------------------------------ async / report
    def set_stream(self, stream):
        """Issue the session's work on a ``torch.cuda.Stream`` (``None``: own stream)."""
        ptr = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        self._check(self.lib.rtr_set_stream(self.handle, ptr))

    def launch_device(self, ids_dev, length):
        """Enqueue one request whose prompt already sits in device memory."""
        self._check(self.lib.rtr_launch(self.handle, ctypes.c_void_p(ids_dev.data_ptr()), length, 1))

    def wait(self):
        self._check(self.lib.rtr_wait(self.handle, ctypes.byref(self._result)))
        return self._record()

    def report(self):
        r = _native.ReportC()
        self._check(self.lib.rtr_get_report(self.handle, ctypes.byref(r)))
        return r.as_dict()

    def profile_gemms(self, rows, reps=5):
        """Average device ms of one pass over every projection GEMM at ``rows`` rows."""
        ms = ctypes.c_float()
        self._check(self.lib.rtr_profile_gemms(self.handle, rows, reps, ctypes.byref(ms)))
        return ms.value
