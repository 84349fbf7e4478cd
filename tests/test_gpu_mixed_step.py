"""The packed engine tick (one forward pass for prefill chunks and decodes together)
against hayate's own model forward, with hayate's model code from ``baseline/_ref``
(skipped where the reference is not installed). Random-init Qwen3-4B weights."""

from __future__ import annotations

import os
import sys

import pytest
import torch

from hayate_b200 import PagedKVCacheManager
from hayate_b200.mixed_step import DecodeGraphs, mixed_generate, packed_forward

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def model():
    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from hayate.model import Qwen3Model

    torch.manual_seed(0)
    with torch.device("cuda"):
        m = Qwen3Model()
    m.initialize_rope("cuda")
    return m.eval()


def manager_for(m, requests=8):
    return PagedKVCacheManager(m.num_layers, m.num_kv_groups, m.head_dim, 64 * 128, 128, requests,
                               torch.bfloat16, "cuda")


def test_packed_forward_matches_model_forward(model):
    """Mixed batch (two prompt chunks of different lengths, two decodes) vs the model's own
    forward on each request alone, with the same history in the pages."""
    gen = torch.Generator(device="cuda").manual_seed(1)
    prompts = [torch.randint(0, 151936, (n,), generator=gen, device="cuda") for n in (300, 77, 40, 9)]
    chunk = [300, 77, 1, 1]   # requests 2 and 3 first prefill all but one token, then decode it
    scores = {}
    for mode in ("packed", "alone"):
        mgr = manager_for(model)
        hs = [mgr.allocate() for _ in prompts]
        with torch.inference_mode():
            for h, p, c in zip(hs, prompts, chunk):   # histories of the decoding requests
                if c == 1:
                    b = mgr.begin_batch([h], len(p) - 1)
                    model(p[None, :-1], paged_cache=b)
                    mgr.commit_batch([h], len(p) - 1)
            new = [p if c > 1 else p[-1:] for p, c in zip(prompts, chunk)]
            if mode == "packed":
                lens = [len(t) for t in new]
                batch = mgr.begin_batch(hs, lens)
                rows = torch.tensor(lens, device="cuda").cumsum(0) - 1
                scores[mode] = packed_forward(model, torch.cat(new), batch, rows).float()
            else:
                outs = []
                for h, t in zip(hs, new):
                    b = mgr.begin_batch([h], len(t))
                    outs.append(model(t[None], paged_cache=b)[0][0, -1].float())
                scores[mode] = torch.stack(outs)
        torch.cuda.synchronize()
        mgr.check_device_errors()
    a, b = scores["packed"], scores["alone"]
    scale = b.abs().max().item()
    err = (a - b).abs().max().item()
    assert err <= 0.05 * scale, (err, scale)
    assert (a.argmax(-1) == b.argmax(-1)).float().mean().item() >= 0.75


def make_engine(model, max_batch=6):
    from hayate.engine import engine as ref_engine
    from hayate.engine.sampler import Sampler
    from hayate.engine.scheduler import Scheduler

    class _Tok:
        eos_token_id = None

        def encode(self, text):
            return [1]

        def decode(self, ids, skip_special_tokens=True):
            return ""

    eng = ref_engine.Engine.__new__(ref_engine.Engine)
    eng.prefill_chunk_size = 128
    eng.model = model
    eng.num_layers, eng.num_kv_groups, eng.head_dim = model.num_layers, model.num_kv_groups, model.head_dim
    eng.max_position_embeddings = model.max_position_embeddings
    eng.tokenizer = _Tok()
    eng.stop_token_ids = set()
    eng.scheduler = Scheduler(max_batch_size=max_batch)
    eng.prefix_cache = None
    eng.sampler = Sampler(eng.tokenizer, set())
    eng.paged_cache = manager_for(model, requests=max_batch)
    return eng


def submit(eng, lengths, max_tokens, seed=2):
    from hayate.engine.request import Request

    gen = torch.Generator().manual_seed(seed)
    reqs = []
    for i, n in enumerate(lengths):
        r = Request(id=i, prompt_tokens=torch.randint(0, 151936, (n,), generator=gen).tolist(), max_tokens=max_tokens)
        eng._prepare_request(r)
        eng.scheduler.add(r)
        reqs.append(r)
    return reqs


@pytest.mark.parametrize("use_graphs", [False, True], ids=["eager", "graphs"])
def test_mixed_generate_runs_requests_to_completion(model, use_graphs):
    eng = make_engine(model)
    graphs = DecodeGraphs(eng, sizes=(4, 8), kv_buckets=(1024,)) if use_graphs else None
    reqs = submit(eng, (5, 300, 129, 1, 700, 64, 33, 250), 6)
    ticks = 0
    with torch.inference_mode():
        while mixed_generate(eng, graphs):
            ticks += 1
            assert ticks < 200
    torch.cuda.synchronize()
    eng.paged_cache.check_device_errors()
    assert all(r.is_completed and len(r.tokens) == 6 for r in reqs)
    held = 1 if use_graphs else 0  # the padding rows' scratch page stays with the manager
    assert len(eng.paged_cache._free_pages) == eng.paged_cache.num_pages - held
    if use_graphs:
        assert graphs.graphs, "no decode tick was replayed from a graph"


def test_decode_graph_matches_eager_forward(model):
    """A graph-replayed decode step (padded to its bucket) scores like the eager packed pass."""
    eng = make_engine(model, max_batch=6)
    reqs = submit(eng, (40, 300, 129, 7, 500), 50, seed=5)
    with torch.inference_mode():
        while any(r.is_prefill for r in reqs):
            mixed_generate(eng)
        decode = [r for r in reqs if not r.is_completed]
        handles = [r.paged_cache for r in decode]
        n = len(decode)
        tokens = torch.tensor([r.tokens[-1] for r in decode], device="cuda")
        batch = eng.paged_cache.begin_batch(handles, [1] * n)
        eager = packed_forward(model, tokens, batch, torch.arange(n, device="cuda")).float()
        graphs = DecodeGraphs(eng, sizes=(8,), kv_buckets=(2048,))
        graph, static, tok_buf, host_tokens, logits, _ = graphs._graph(n, max(h.length for h in handles) + 1)
        host_tokens.zero_()
        host_tokens[:n] = tokens.cpu()
        static.update(handles)
        tok_buf.copy_(host_tokens)
        graph.replay()
        replayed = logits[:n].float()
        torch.cuda.synchronize()
    eng.paged_cache.check_device_errors()
    scale = eager.abs().max().item()
    assert (replayed - eager).abs().max().item() <= 0.05 * scale
    assert (replayed.argmax(-1) == eager.argmax(-1)).float().mean().item() >= 0.75
