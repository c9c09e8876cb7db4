"""CPU restatement of one request of the reference's constrained beam search.

The loop is ``transformers`` 5.5.0 ``GenerationMixin._beam_search``
(``generation/utils.py``; the reference pins 4.55.4 whose vectorised helpers
are the same), specialised to what the reference runs
(``benchmark_inference.py:139-146``): batch 1, ``num_beams=50``,
``num_return_sequences=50``, ``max_new_tokens=8``, ``length_penalty=0``,
``early_stopping=False``, greedy beams, one EOS id, ``output_scores=True``.
Torch ops are used in the same order so the CPU result is bit-identical:

* init: ``running_beam_scores[:, 1:] = -1e9``, finished scores -1e9 (utils.py:3196-3204);
* step: ``log_softmax(float(logits))`` then the processor (:3252-3257);
  processor = ``GpuSidConstrainedLogitsProcessor.__call__``
  (``rapidtinyrec/gpu_constraints.py:95-101``): second ``log_softmax``, ``-inf``
  mask with 0 scattered at the allowed columns;
* ``+ running_beam_scores`` and ``_get_top_k_continuations`` with
  ``topk(100)`` (:2945-2997);
* EOS stopping criterion, ``_get_running_beams_for_next_iteration`` (:2999-3019);
* ``_update_finished_beams`` (:3021-3072);
* cache reorder by the parent index, ``_check_early_stop_heuristic`` and
  ``_beam_search_has_unfinished_sequences`` (:2876-2943, :3347-3372);
* outputs: ``sequences``, ``sequences_scores``, ``beam_indices``, ``scores``
  and ``compute_transition_scores`` (:1335) as unpacked by
  ``benchmark_inference.py:150-154``.
"""
from __future__ import annotations

import numpy as np
import torch

from .sid_tables import semantic_allowed

NUM_BEAMS = 50


def process_scores(log_probs, input_ids, constraints, eos_id, step, tables=None):
    """``GpuSidConstrainedLogitsProcessor.__call__`` on ``[rows, V]`` log-probs."""
    scores = torch.nn.functional.log_softmax(log_probs, dim=-1)
    mask = torch.full_like(scores, float('-inf'))
    if tables is not None:
        columns = torch.as_tensor(tables.lookup(step, input_ids.numpy()), dtype=torch.long)
    else:
        rows = [semantic_allowed(constraints, eos_id, step, r) for r in input_ids.tolist()]
        width = max(len(r) for r in rows)
        columns = torch.tensor([r + [r[0]] * (width - len(r)) for r in rows], dtype=torch.long)
    mask.scatter_(1, columns, 0.0)
    return scores + mask


def beam_search(model, prompt_ids, constraints, eos_id, pad_id=None, num_beams=NUM_BEAMS,
                max_new_tokens=8, tables=None, on_step=None):
    """Run one request; returns the reference's per-request output record.

    ``model`` provides ``prefill(ids) -> (logits[1,V], cache)``,
    ``decode(tokens, position, cache) -> logits[B,V]`` and ``reorder(cache, idx)``.
    """
    pad_id = eos_id if pad_id is None else pad_id
    prompt = torch.as_tensor(prompt_ids, dtype=torch.long)
    cur_len = decoder_prompt_len = prompt.shape[0]
    max_length = cur_len + max_new_tokens
    beams_to_keep = 2 * num_beams
    top_num_beam_mask = torch.cat((torch.ones(num_beams, dtype=torch.bool),
                                   torch.zeros(beams_to_keep - num_beams, dtype=torch.bool)))
    running_sequences = torch.full((1, num_beams, max_length), pad_id, dtype=torch.int64)
    running_sequences[:, :, :cur_len] = prompt
    sequences = running_sequences.clone()
    running_beam_scores = torch.zeros((1, num_beams), dtype=torch.float)
    running_beam_scores[:, 1:] = -1e9
    beam_scores = torch.full((1, num_beams), -1e9, dtype=torch.float)
    is_sent_finished = torch.zeros((1, num_beams), dtype=torch.bool)
    unsatisfied = torch.ones((1, 1), dtype=torch.bool)
    running_beam_indices = torch.full((1, num_beams, max_length - cur_len), -1, dtype=torch.int32)
    beam_indices = running_beam_indices.clone()
    all_scores = []

    logits, cache = model.prefill(prompt)
    logits = logits.repeat_interleave(num_beams, dim=0)      # PrefillOnce: shared_prefill.py:57
    step = 0
    finished = False
    while not finished:
        if step:
            flat = running_sequences[0, :, :cur_len]
            logits = model.decode(flat[:, -1], cur_len - 1, cache)
        flat_running = running_sequences[0, :, :cur_len]
        log_probs = torch.nn.functional.log_softmax(logits.to(dtype=torch.float32), dim=-1)
        log_probs = process_scores(log_probs, flat_running, constraints, eos_id, step, tables)
        all_scores.append(log_probs.clone())
        vocab = log_probs.shape[-1]
        acc = (log_probs[None] + running_beam_scores[:, :, None]).reshape(1, num_beams * vocab)

        # _get_top_k_continuations
        topk_log_probs, topk_indices = torch.topk(acc, k=beams_to_keep)
        topk_beam = topk_indices // vocab
        topk_sequences = torch.take_along_dim(running_sequences, topk_beam[..., None], dim=1)
        topk_beam_indices = torch.take_along_dim(running_beam_indices, topk_beam[..., None], dim=1)
        topk_ids = topk_indices % vocab
        topk_sequences[:, :, cur_len] = topk_ids
        topk_beam_indices[:, :, cur_len - decoder_prompt_len] = topk_beam.to(torch.int32)

        # EOS + max-length stopping criteria on the candidate sequences
        hits = topk_ids == eos_id
        if cur_len + 1 >= max_length:
            hits = torch.ones_like(hits)

        # _get_running_beams_for_next_iteration
        topk_running = topk_log_probs + hits.to(torch.float32) * -1.0e9
        nxt = torch.topk(topk_running, k=num_beams)[1]
        running_sequences = torch.take_along_dim(topk_sequences, nxt[..., None], dim=1)
        running_beam_scores = torch.take_along_dim(topk_running, nxt, dim=1)
        running_beam_indices = torch.take_along_dim(topk_beam_indices, nxt[..., None], dim=1)

        # _update_finished_beams (length_penalty=0, early_stopping=False)
        did_finish = hits & top_num_beam_mask[None, :]
        fin = topk_log_probs / ((cur_len + 1 - decoder_prompt_len) ** 0.0)
        full = torch.all(is_sent_finished, dim=-1, keepdim=True) & False
        fin = fin + full.to(torch.float32) * -1.0e9
        fin = fin + (~unsatisfied).to(torch.float32) * -1.0e9
        fin = fin + (~did_finish) * -1.0e9
        merged_seq = torch.cat((sequences, topk_sequences), dim=1)
        merged_scores = torch.cat((beam_scores, fin), dim=1)
        merged_idx = torch.cat((beam_indices, topk_beam_indices), dim=1)
        merged_done = torch.cat((is_sent_finished, did_finish), dim=1)
        keep = torch.topk(merged_scores, k=num_beams)[1]
        sequences = torch.take_along_dim(merged_seq, keep[..., None], dim=1)
        beam_scores = torch.take_along_dim(merged_scores, keep, dim=1)
        beam_indices = torch.take_along_dim(merged_idx, keep[..., None], dim=1)
        is_sent_finished = torch.take_along_dim(merged_done, keep, dim=1)

        # reorder the cache by the parents of the new running beams
        parents = running_beam_indices[0, :, cur_len - decoder_prompt_len]
        model.reorder(cache, parents.to(torch.long))
        if on_step is not None:
            on_step(step, log_probs, topk_log_probs, topk_indices, parents)

        cur_len += 1
        best_running = running_beam_scores[:, :1] / ((cur_len - decoder_prompt_len) ** 0.0)
        worst_finished = torch.where(is_sent_finished, torch.min(beam_scores, dim=1, keepdim=True)[0], -1.0e9)
        unsatisfied = unsatisfied & torch.any(best_running > worst_finished, dim=-1, keepdim=True)
        has_unfinished = bool(torch.any(unsatisfied)) and not bool(torch.all(hits))
        finished = not has_unfinished
        step += 1

    # outputs (utils.py:3375-3387)
    max_generated = int(((beam_indices[0] + 1).bool()).sum(dim=1).max())
    seqs = sequences[0, :, :decoder_prompt_len + max_generated]
    bidx = beam_indices[0, :, :max_generated]
    token_ids = seqs[:, decoder_prompt_len:]
    trans = torch.stack([all_scores[t][bidx[:, t].long(), token_ids[:, t]] for t in range(max_generated)], dim=1)
    return {
        'steps': step,
        'beam_indices': bidx.tolist(),
        'score_dtypes': [str(s.dtype) for s in all_scores],
        'token_ids': token_ids.tolist(),
        'sequence_logp': beam_scores[0].float().tolist(),
        'transition_logp': trans.float().tolist(),
        'scores': all_scores,
    }


def sparse_scores(scores):
    """Finite entries of each step's processed scores: (rows, cols, values) arrays."""
    out = []
    for s in scores:
        rows, cols = torch.nonzero(torch.isfinite(s), as_tuple=True)
        out.append((rows.numpy().astype(np.int32), cols.numpy().astype(np.int32),
                    s[rows, cols].numpy().astype(np.float32)))
    return out
