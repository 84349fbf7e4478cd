"""One engine tick as packed forward passes: prefill chunks and decodes together.

hayate's ``Engine.generate`` (``hayate/engine/engine.py:291-314``) runs, each scheduler
tick, one forward pass per group of up to ``MAX_PREFILL_BATCH`` prompts *per distinct
chunk length* (``prefill_batch``, ``engine.py:226-283``: "equal-length groups avoid
padded writes into physical pages") and then one more pass for every decoding request
(``decode_batch``, ``engine.py:285-296``). Each pass reads all of the model's weights.

``mixed_generate`` keeps that tick's semantics (same scheduler, same chunking of
prompts, same sampler calls and ``finalize`` order, prompts finishing in a tick start
decoding the next one) but puts each group of up to ``MAX_PREFILL_BATCH`` prompt
chunks, whatever their lengths, and in the first group every decoding request's one
token, into ONE packed batch (``PagedKVCacheManager.begin_batch`` with one query length
per request): one forward pass where the reference runs several. The model's own
modules run unchanged on the ``[1, N, hidden]`` token axis; per layer, QK-norm + RoPE +
``write_layer`` is one fused launch (``PagedKVBatch.prepare_layer``, positions from the
batch's own metadata) and ``attend_layer`` serves the decode rows and the prefill rows
in one call. Only rows that sample go through the final norm and output head.
"""

from __future__ import annotations

import torch

from .paged_cache import PagedKVBatch

MAX_PREFILL_BATCH = 8  # hayate/engine/constants.py:11


def packed_forward(model, token_ids: torch.Tensor, batch: PagedKVBatch,
                   sample_rows: torch.Tensor) -> torch.Tensor:
    """Run ``model`` (a hayate ``Qwen3Model``) over a packed batch's tokens.

    ``token_ids`` is ``[N]`` (the batch's token axis), ``sample_rows`` the rows whose
    next-token scores are wanted. Returns ``[len(sample_rows), vocab]`` scores, computed
    like ``Qwen3Model.forward`` (``hayate/model/qwen.py:69-175`` with
    ``block.py`` / ``attention.py``) for those rows.
    """
    n = token_ids.numel()
    x = model.embed_tokens(token_ids).unsqueeze(0)
    for layer_idx, block in enumerate(model.layers):
        attn = block.self_attn
        shortcut = x
        h = block.input_layernorm(x)
        q = attn.q_proj(h).view(1, n, attn.num_heads, attn.head_dim)
        k = attn.k_proj(h).view(1, n, attn.num_kv_groups, attn.head_dim)
        v = attn.v_proj(h).view(1, n, attn.num_kv_groups, attn.head_dim)
        eps = attn.q_norm.eps if attn.q_norm.eps is not None else 1e-6
        q = batch.prepare_layer(layer_idx, q, k, v, attn.q_norm.weight, attn.k_norm.weight,
                                model.cos, model.sin, eps)
        context = batch.attend_layer(q, layer_idx).transpose(1, 2).reshape(1, n, -1)
        x = attn.o_proj(context) + shortcut
        shortcut = x
        x = block.mlp(block.post_attention_layernorm(x)) + shortcut
    return model.out_head(model.norm(x[0, sample_rows]))


def _prompt_chunk(engine, request):
    """The next prompt chunk of ``request`` (``engine.py:229-256``): (tokens, completes)."""
    if not request.prompt_tokens:
        request.prompt_tokens = engine.tokenizer.encode(request.prompt)
    if not request.prompt_tokens:
        raise ValueError("prompt must tokenize to at least one token")
    max_prefix_len = len(request.prompt_tokens) - 1
    if request.paged_cache is None:
        request.paged_cache = engine.paged_cache.allocate_for_request(request.kv_cache)
        if request.kv_cache is not None:
            request.kv_cache.reset()
            request.kv_cache = None
    cache_pos = request.paged_cache.length
    if cache_pos > max_prefix_len:
        engine.paged_cache.truncate(request.paged_cache, max_prefix_len)
        cache_pos = max_prefix_len
    end = min(cache_pos + engine.prefill_chunk_size, len(request.prompt_tokens))
    return request.prompt_tokens[cache_pos:end], end == len(request.prompt_tokens)


def _run_group(engine, prefill, decode, device):
    """One packed forward pass over ``prefill`` chunks and ``decode`` tokens."""
    requests, tokens, lengths, sampled = [], [], [], []
    for request in prefill:
        chunk, completes = _prompt_chunk(engine, request)
        requests.append(request)
        tokens.extend(chunk)
        lengths.append(len(chunk))
        sampled.append(completes)
    for request in decode:
        if request.paged_cache is None:
            raise RuntimeError("every request must own paged KV storage before inference")
        requests.append(request)
        tokens.append(request.tokens[-1])
        lengths.append(1)
        sampled.append(True)
    handles = [request.paged_cache for request in requests]
    batch = engine.paged_cache.begin_batch(handles, lengths)
    ends = torch.tensor(lengths, dtype=torch.long).cumsum(0) - 1
    rows = [i for i, s in enumerate(sampled) if s]
    token_ids = torch.tensor(tokens, dtype=torch.long, device=device)
    with torch.inference_mode():
        logits = packed_forward(engine.model, token_ids, batch, ends[rows].to(device))
    engine.paged_cache.commit_batch(handles, lengths)
    if not rows:
        return
    chosen = [requests[i] for i in rows]
    next_tokens = engine.sampler.sample(logits, chosen).flatten().tolist()
    n_prefill = len(prefill)
    for i, request, token in zip(rows, chosen, next_tokens):
        engine.sampler.finalize(request, token)
        if i < n_prefill:  # a prompt finished this tick: it decodes from the next one
            request.is_prefill = False
            engine._store_prompt_prefix(request)


def mixed_generate(engine) -> bool:
    """Run one scheduler tick of ``engine`` (a hayate ``Engine`` whose ``paged_cache`` is a
    ``hayate_b200.PagedKVCacheManager``) with packed forward passes; return whether any
    request remains active (``Engine.generate``'s contract)."""
    previous = list(engine.scheduler.current_batch)
    batch = engine.scheduler.tick()
    active = {id(request) for request in batch}
    for request in previous:
        if request.is_completed and id(request) not in active:
            engine.release_request_cache(request)
    if not batch:
        return False
    prefill = [r for r in batch if r.is_prefill]
    decode = [r for r in batch if not r.is_prefill]
    device = engine.paged_cache.device
    groups = [prefill[i:i + MAX_PREFILL_BATCH] for i in range(0, len(prefill), MAX_PREFILL_BATCH)] or [[]]
    for index, group in enumerate(groups):
        _run_group(engine, group, decode if index == 0 else [], device)
    return True
