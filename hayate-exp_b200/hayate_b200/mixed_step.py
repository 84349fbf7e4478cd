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


class DecodeGraphs:
    """Decode-only ticks replayed from CUDA graphs.

    Once every active request is decoding, a tick is the same short forward pass over a
    few dozen tokens; run eagerly, its ~20 launches per layer cost more host time than the
    GPU needs. Here each (batch size bucket, longest-context bucket) gets one graph of
    ``packed_forward`` over a ``StaticDecodeBatch`` (captured on first use); a tick copies
    the tokens and the page metadata into the graph's buffers and replays it. Requests
    beyond the real batch are padding rows on the manager's scratch page, their scores
    discarded. Sampling, ``finalize`` and the page bookkeeping are ``decode_batch``'s
    (``engine.py:285-296``).
    """

    def __init__(self, engine, sizes=(8, 16, 32, 48, 64, 96, 128),
                 kv_buckets=(2048, 4096, 8192, 16384, 32768)):
        self.engine = engine
        manager = engine.paged_cache
        limit = min(manager.capacity_tokens, engine.max_position_embeddings)
        self.sizes = sorted({n for n in sizes if n < manager.max_requests} | {manager.max_requests})
        self.kv_buckets = sorted({min(k, limit) for k in kv_buckets} | {limit})
        self.graphs: dict = {}
        self.device = manager.device

    def _graph(self, n: int, max_kv: int):
        size = next((s for s in self.sizes if s >= n), None)
        kv = next((k for k in self.kv_buckets if k >= max_kv), None)
        if size is None or kv is None:
            return None
        key = (size, kv)
        if key not in self.graphs:
            self.graphs[key] = self._capture(size, kv)
        return self.graphs[key]

    def _capture(self, size: int, kv: int):
        model = self.engine.model
        static = self.engine.paged_cache.static_decode_batch(size, kv, model.layers[0].self_attn.num_heads)
        tokens = torch.zeros(size, dtype=torch.long, device=self.device)
        rows = torch.arange(size, device=self.device)
        host_tokens = torch.zeros(size, dtype=torch.long, pin_memory=True)
        static.update([])  # all padding while capturing
        with torch.inference_mode():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):  # warm-up outside the capture (library set-up)
                for _ in range(2):
                    packed_forward(model, tokens, static.batch, rows)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                logits = packed_forward(model, tokens, static.batch, rows)
        # every tensor the graph reads must outlive it: rows is kept with the graph
        return graph, static, tokens, host_tokens, logits, rows

    def step(self, decode) -> bool:
        """Run one decode tick for ``decode`` from a graph; False if no bucket fits."""
        handles = [request.paged_cache for request in decode]
        if any(h is None for h in handles):
            raise RuntimeError("every request must own paged KV storage before inference")
        n = len(decode)
        found = self._graph(n, max(h.length for h in handles) + 1)
        if found is None:
            return False
        graph, static, tokens, host_tokens, logits, _ = found
        torch.cuda.current_stream().synchronize()  # the pinned token buffer is reused
        host_tokens.zero_()
        host_tokens[:n] = torch.tensor([request.tokens[-1] for request in decode])
        static.update(handles)
        tokens.copy_(host_tokens, non_blocking=True)
        graph.replay()
        self.engine.paged_cache.commit_batch(handles, 1)
        next_tokens = self.engine.sampler.sample(logits[:n], decode).flatten().tolist()
        for request, token in zip(decode, next_tokens):
            self.engine.sampler.finalize(request, token)
        return True


def mixed_generate(engine, graphs: DecodeGraphs | None = None) -> bool:
    """Run one scheduler tick of ``engine`` (a hayate ``Engine`` whose ``paged_cache`` is a
    ``hayate_b200.PagedKVCacheManager``) with packed forward passes; return whether any
    request remains active (``Engine.generate``'s contract). With ``graphs``, ticks in which
    every request decodes replay a CUDA graph."""
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
    if graphs is not None and not prefill and graphs.step(decode):
        return True
    device = engine.paged_cache.device
    groups = [prefill[i:i + MAX_PREFILL_BATCH] for i in range(0, len(prefill), MAX_PREFILL_BATCH)] or [[]]
    for index, group in enumerate(groups):
        _run_group(engine, group, decode if index == 0 else [], device)
    return True
