"""GPU parity: the CUDA kernels against the reference's golden vectors and the oracle.

Tolerances (max-abs on attention outputs): 2e-2 for bf16/f16, 1e-4 for f32.
The scatter is compared bit for bit (SHA-256 of the whole pool).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from golden_util import CASES, load_golden, make_inputs, sha256_f32, shuffled_free_pages
from hayate_b200 import Cache, PagedKVCacheManager, ops
from hayate_b200 import workloads as W

import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}


def golden_run(case, dtype, kernel="auto", split_tokens=0):
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    manager = PagedKVCacheManager(case.num_layers, case.num_kv_heads, case.head_dim,
                                  case.max_cache_tokens, case.page_size, case.batch, dtype, "cuda")
    manager.kernel, manager.split_tokens = kernel, split_tokens
    manager._free_pages = shuffled_free_pages(manager.num_pages, case.seed)
    handles = []
    for hk, hv in zip(inputs["hist_k"], inputs["hist_v"]):
        cache = Cache.from_tensors(torch.from_numpy(hk), torch.from_numpy(hv)) if hk.shape[2] else None
        handles.append(manager.allocate_for_request(cache))
    batch = manager.begin_batch(handles, case.query_len)
    dev = lambda a: torch.from_numpy(a).to("cuda", dtype)  # noqa: E731
    batch.write_layer(case.layer, dev(inputs["k_new"]), dev(inputs["v_new"]))
    out = batch.attend_layer(dev(inputs["q"]), case.layer)
    torch.cuda.synchronize()
    manager.check_device_errors()
    return manager, out, golden


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=str)
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_golden_case(case, dtype):
    manager, out, golden = golden_run(case, dtype)
    assert sha256_f32(manager.k_cache.float().cpu().numpy()) == str(golden["k_pool_sha256"])
    assert sha256_f32(manager.v_cache.float().cpu().numpy()) == str(golden["v_pool_sha256"])
    err = (out.float().cpu() - torch.from_numpy(golden["out"])).abs().max().item()
    assert err <= TOL[dtype], err


@pytest.mark.parametrize("kernel", ["generic", "decode"])
def test_golden_decode_case_each_kernel(kernel):
    case = [c for c in CASES if c.name == "qwen_decode"][0]
    for split in (0, 64, 128):
        _, out, golden = golden_run(case, torch.bfloat16, kernel=kernel, split_tokens=split)
        err = (out.float().cpu() - torch.from_numpy(golden["out"])).abs().max().item()
        assert err <= 2e-2, (split, err)


def build_step(lengths, query_len, dtype=torch.bfloat16, seed=0, page_size=128, num_layers=1,
               layer=0, slack_pages=2, strided=True):
    """A manager holding synthetic histories, one step's inputs and its batch."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    pages = sum(math.ceil((n + query_len) / page_size) for n in lengths) + slack_pages
    manager = PagedKVCacheManager(num_layers, 8, 128, pages * page_size, page_size,
                                  len(lengths), dtype, "cuda")
    W.shuffle_free_pages(manager, seed)
    handles = [manager.allocate() for _ in lengths]
    for h, n in zip(handles, lengths):
        W.fill_history(manager, h, n, gen, layers=[layer])
    q, k, v = W.step_inputs(manager, handles, query_len, 32, gen, strided=strided)
    batch = manager.begin_batch(handles, query_len)
    return manager, handles, batch, q, k, v


def oracle_out(manager, batch, q, layer=0, requests=None):
    kp = manager.k_cache.float().cpu().numpy()
    vp = manager.v_cache.float().cpu().numpy()
    table = batch.page_table.cpu().numpy().astype(np.int64)
    lens = batch.cache_lens.cpu().numpy()
    return oracle.paged_attention(q.float().cpu().numpy(), kp, vp, layer, table, lens,
                                  manager.page_size, requests=requests)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("query_len", [1, 2, 3, 4])
@pytest.mark.parametrize("split", [0, 64, 192, 1024])
def test_decode_kernel_matches_oracle(query_len, split, dtype):
    lengths = [0, 1, 63, 64, 127, 128, 1000, 2431]
    manager, _, batch, q, k, v = build_step(lengths, query_len, dtype=dtype, seed=query_len)
    manager.kernel, manager.split_tokens = "decode", split
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    manager.check_device_errors()
    ref = oracle_out(manager, batch, q)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= 2e-2, err


def test_decode_is_deterministic_and_leaves_counters_zero():
    manager, _, batch, q, k, v = build_step([3000, 5000, 70], 1, seed=3)
    manager.kernel, manager.split_tokens = "decode", 256
    batch.write_layer(0, k, v)
    first = batch.attend_layer(q, 0).clone()
    second = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    ws = manager._workspace
    assert ws is not None and int(ws[:256].view(torch.int32).abs().sum()) == 0


def oracle_request_rows(manager, batch, q, requests, layer=0):
    """The oracle's rows for some requests, each computed on a compact copy of only that
    request's pages (host memory stays bounded at full config sizes)."""
    table = batch.page_table.cpu().numpy().astype(np.int64)
    lens = batch.cache_lens.cpu().numpy()
    P, T = manager.page_size, q.shape[2]
    H, D = manager.num_kv_heads, manager.head_dim
    rows = {}
    for b in requests:
        n = -(-(int(lens[b]) + T) // P)
        pages = torch.from_numpy(table[b, :n]).to(q.device)
        pools = []
        for pool in (manager.k_cache, manager.v_cache):
            paged = pool[layer, 0].view(H, manager.num_pages, P, D)
            pools.append(paged.index_select(1, pages).reshape(1, 1, H, n * P, D).float().cpu().numpy())
        rows[b] = oracle.paged_attention(q[b:b + 1].float().cpu().numpy(), pools[0], pools[1], 0,
                                         np.arange(n, dtype=np.int64)[None], lens[b:b + 1], P)[0]
    return rows


def test_full_size_decode_sweep_config():
    """Config 2 shapes (B=64, kv 1024..8192, shuffled pages): every request against the oracle,
    through the one-launch decode step (the kernel writes the new rows itself)."""
    rng = np.random.RandomState(0)
    lengths = [int(n) - 1 for n in rng.randint(1024, 8193, size=64)]
    manager, _, batch, q, k, v = build_step(lengths, 1, seed=11)
    out = batch.write_attend_layer(0, k, v, q)
    torch.cuda.synchronize()
    manager.check_device_errors()
    got = out.float().cpu().numpy()
    ref = oracle_request_rows(manager, batch, q, range(64))
    err = max(float(np.abs(got[b] - ref[b]).max()) for b in range(64))
    assert err <= 2e-2, err
    # the rows the step wrote are the step's k/v, bit for bit
    table, lens = batch.page_table.long(), batch.cache_lens
    slots = table[torch.arange(64, device="cuda"), lens // 128] * 128 + lens % 128
    assert torch.equal(manager.k_cache[0, 0][:, slots], k[:, :, 0].transpose(0, 1))
    assert torch.equal(manager.v_cache[0, 0][:, slots], v[:, :, 0].transpose(0, 1))


@pytest.mark.parametrize("query_len", [1, 7, 130])
def test_generic_kernel_f32_matches_oracle(query_len):
    manager, _, batch, q, k, v = build_step([0, 200, 513], query_len, dtype=torch.float32, seed=5)
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    ref = oracle_out(manager, batch, q)
    err = np.abs(out.cpu().numpy() - ref).max()
    assert err <= 1e-4, err


def test_scatter_contiguous_and_strided_inputs_agree():
    lengths = [5, 300]
    outs = []
    for strided in (True, False):
        manager, _, batch, q, k, v = build_step(lengths, 3, seed=9, strided=strided)
        batch.write_layer(0, k, v)
        torch.cuda.synchronize()
        outs.append((manager.k_cache.clone(), manager.v_cache.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_kernels_flag_bad_page_ids_without_touching_memory():
    """A page id past the pool is refused by the kernels' own range checks (error word set)."""
    manager, _, batch, q, k, v = build_step([300], 1, seed=2)
    table = batch.page_table.clone()
    table[0, 2] = manager.num_pages + 5  # the new token's page: refused before any access
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    before = manager.k_cache.clone()
    ops.kv_scatter(k, v, manager.k_cache, manager.v_cache, 0, table, batch.cache_lens_i32,
                   manager.page_size, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1 and torch.equal(before, manager.k_cache)
    for kernel in ("decode", "generic"):
        err.zero_()
        ws = ops.new_workspace(ops.attention_workspace_bytes(1, 1, 32, 8, 128, 301, q.dtype, 64), "cuda")
        ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, table, batch.cache_lens_i32,
                            manager.page_size, 301, workspace=ws, error_word=err, kernel=kernel,
                            split_tokens=64)
        torch.cuda.synchronize()
        assert int(err.item()) & 1, kernel


AUTO_SPLIT_CASES = [
    ([10, 20], 8192),            # a grid sized for 8192 keys: most splits have nothing to do
    ([30000], 0),                # one request: many splits per (request, head)
    ([0, 1, 63, 64, 127, 128, 1000, 2431], 0),   # empty history, page edges
    ([4096] * 3 + [5, 9000, 77], 16384),         # long and short requests, slack in max_kv_len
]


@pytest.mark.parametrize("lengths, max_kv", AUTO_SPLIT_CASES, ids=str)
def test_auto_split_decode_matches_oracle(lengths, max_kv):
    """The decode step with the library's own split size (split_tokens 0), the fused row write
    and a max_kv_len larger than needed: every request against the oracle, twice (the split
    counters are left zero), on shapes that leave splits idle, cut one request into many
    splits, or mix empty, short and long requests."""
    manager, _, batch, q, k, v = build_step(lengths, 1, seed=len(lengths) + 3)
    max_kv = max(max_kv, batch.max_kv_len)
    need = ops.attention_workspace_bytes(len(lengths), 1, 32, 8, 128, max_kv, q.dtype, 0)
    ws = ops.new_workspace(need, "cuda")
    outs = []
    for _ in range(2):  # a second call: the unit counters were left zero
        outs.append(ops.paged_attention_scatter(q, k, v, manager.k_cache, manager.v_cache, 0,
                                                batch.page_table, batch.cache_lens_i32, 128, max_kv,
                                                workspace=ws, error_word=manager.error_word))
    torch.cuda.synchronize()
    manager.check_device_errors()
    assert torch.equal(outs[0], outs[1])
    if need:  # the split counters sit at the workspace's start and are left zero
        assert int(ws[: len(lengths) * 8 * 4].view(torch.int32).abs().sum()) == 0
    got = outs[0].float().cpu().numpy()
    ref = oracle_request_rows(manager, batch, q, range(len(lengths)))
    err = max(float(np.abs(got[b] - ref[b]).max()) for b in range(len(lengths)))
    assert err <= 2e-2, err


def test_auto_split_decode_flags_a_bad_page_and_recovers():
    """A page id outside the pool in the middle of a long request: the decode kernel flags
    it, the split that holds it loads nothing, the counters are left zero and the next clean
    call matches the oracle."""
    manager, _, batch, q, k, v = build_step([9000, 300], 1, seed=6)
    batch.write_layer(0, k, v)
    table = batch.page_table.clone()
    table[0, 30] = manager.num_pages + 3
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = ops.new_workspace(ops.attention_workspace_bytes(2, 1, 32, 8, 128, batch.max_kv_len, q.dtype, 0), "cuda")
    ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, table, batch.cache_lens_i32, 128,
                        batch.max_kv_len, workspace=ws, error_word=err)
    torch.cuda.synchronize()
    assert ops.read_device_errors(err) == ["page id outside the pool"]
    assert int(ws[:64].view(torch.int32).abs().sum()) == 0  # counters still left zero
    good = ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, batch.page_table,
                               batch.cache_lens_i32, 128, batch.max_kv_len, workspace=ws,
                               error_word=manager.error_word)
    torch.cuda.synchronize()
    manager.check_device_errors()
    ref = oracle_request_rows(manager, batch, q, [0, 1])
    assert max(float(np.abs(good.float().cpu().numpy()[b] - ref[b]).max()) for b in (0, 1)) <= 2e-2


def test_attend_output_layout_is_transpose_friendly():
    manager, _, batch, q, k, v = build_step([10, 20], 1, seed=1)
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    assert out.shape == q.shape
    assert out.transpose(1, 2).is_contiguous()


PREFILL_CASES = [
    ([0], 1), ([0, 5], 5), ([127, 128, 129], 128), ([0, 200, 1000], 130),
    ([4095, 33], 512), ([1, 2048], 257), ([300], 1000),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("lengths, query_len", PREFILL_CASES, ids=str)
def test_prefill_kernel_matches_oracle(lengths, query_len, dtype):
    manager, _, batch, q, k, v = build_step(lengths, query_len, dtype=dtype, seed=len(lengths) + query_len)
    manager.kernel = "prefill"
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    manager.check_device_errors()
    ref = oracle_out(manager, batch, q)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= 2e-2, err


@pytest.mark.parametrize("page_size", [256, 512])
def test_prefill_kernel_large_pages(page_size):
    manager, _, batch, q, k, v = build_step([70, 600], 300, page_size=page_size, seed=page_size)
    manager.kernel = "prefill"
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    manager.check_device_errors()
    err = np.abs(out.float().cpu().numpy() - oracle_out(manager, batch, q)).max()
    assert err <= 2e-2, err


def test_prefill_contiguous_q_and_multi_layer():
    gen = torch.Generator(device="cuda").manual_seed(4)
    manager = PagedKVCacheManager(3, 8, 128, 64 * 128, 128, 2, torch.bfloat16, "cuda")
    W.shuffle_free_pages(manager, 4)
    handles = [manager.allocate() for _ in range(2)]
    for h, n in zip(handles, (100, 900)):
        W.fill_history(manager, h, n, gen)
    q, k, v = W.step_inputs(manager, handles, 64, 32, gen, strided=False)
    batch = manager.begin_batch(handles, 64)
    for layer in range(3):
        batch.write_layer(layer, k, v)
    out = batch.attend_layer(q, 2)
    torch.cuda.synchronize()
    manager.check_device_errors()
    err = np.abs(out.float().cpu().numpy() - oracle_out(manager, batch, q, layer=2)).max()
    assert err <= 2e-2, err


@pytest.mark.parametrize("plan", [False, True], ids=["default_grid", "planned"])
def test_full_size_prefill_config(plan):
    """Config 3 shapes (8 requests x 512-token chunk on prefixes U[0, 4096]): every request
    against the oracle, on the default grid and on a planned schedule with items cut in two."""
    rng = np.random.RandomState(1)
    prefixes = [int(n) for n in rng.randint(0, 4097, size=8)]
    manager, _, batch, q, k, v = build_step(prefixes, 512, seed=21)
    if plan:
        # a near-free merge cost makes the planner cut its heaviest items in two
        items, splits = ops.prefill_plan(prefixes, 512, 32, manager.num_sms, 128, item_overhead=5.0,
                                         merge_cost=0.01)
        assert items is not None and splits > 0
    batch.write_layer(0, k, v)
    if plan:
        out = ops.prefill_attention_planned(
            q, manager.k_cache, manager.v_cache, 0, batch.page_table, batch.cache_lens_i32, 128,
            torch.from_numpy(items.reshape(-1)).to("cuda").view(-1, 4), splits,
            workspace=manager.prefill_workspace(splits), error_word=manager.error_word)
    else:
        manager.prefill_plan = False
        out = batch.attend_layer(q, 0)  # auto: the tcgen05 prefill kernel, default grid
    torch.cuda.synchronize()
    manager.check_device_errors()
    got = out.float().cpu().numpy()
    ref = oracle_request_rows(manager, batch, q, range(8))
    err = max(float(np.abs(got[b] - ref[b]).max()) for b in range(8))
    assert err <= 2e-2, err


@pytest.mark.parametrize("column", [0, 1, 2])
def test_prefill_flags_bad_page_ids(column):
    """A page id outside the pool, in the first, a middle or the last key tile: refused by
    the producer when it reaches that tile; the CTA writes zeros and the next call is clean."""
    manager, _, batch, q, k, v = build_step([300], 40, seed=2)
    batch.write_layer(0, k, v)
    table = batch.page_table.clone()
    table[0, column] = -7 if column != 1 else manager.num_pages
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, table, batch.cache_lens_i32,
                              manager.page_size, 340, error_word=err, kernel="prefill")
    torch.cuda.synchronize()
    assert ops.read_device_errors(err) == ["page id outside the pool"]
    assert float(out.float().abs().max()) == 0.0  # refused CTAs write zeros
    err.zero_()
    good = ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, batch.page_table,
                               batch.cache_lens_i32, manager.page_size, 340, error_word=err,
                               kernel="prefill")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.abs(good.float().cpu().numpy() - oracle_out(manager, batch, q)).max() <= 2e-2


def test_prefill_flags_short_page_table():
    """A table row with fewer pages than the kv length needs is refused before any load."""
    manager, _, batch, q, k, v = build_step([300], 40, seed=3)
    table = torch.empty((1, 2), dtype=torch.int32, device="cuda")  # row stride 2: 2 pages,
    table.copy_(batch.page_table[:, :2])                            # 340 keys need 3
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, table, batch.cache_lens_i32,
                              manager.page_size, 340, error_word=err, kernel="prefill")
    torch.cuda.synchronize()
    assert ops.read_device_errors(err) == ["kv length needs more pages than the page table row holds"]
    assert float(out.float().abs().max()) == 0.0


def test_prefill_q_load_paths_agree():
    """Q by TMA (q in [B, H, T, D] or [B, T, H, D] memory) and Q by plain loads (a q
    broadcast over the batch, which no tensor map describes) give identical rows."""
    manager, _, batch, q, k, v = build_step([0, 700, 129], 300, seed=8)
    batch.write_layer(0, k, v)
    one = q[:1]
    broadcast = one.expand(3, -1, -1, -1)                         # b stride 0: plain loads
    contiguous = broadcast.contiguous()                           # (d, t, h, b) map
    transposed = broadcast.transpose(1, 2).contiguous().transpose(1, 2)  # (d, h, t, b) map
    outs = []
    for qq in (broadcast, contiguous, transposed):
        outs.append(ops.paged_attention(qq, manager.k_cache, manager.v_cache, 0, batch.page_table,
                                        batch.cache_lens_i32, manager.page_size, batch.max_kv_len,
                                        error_word=manager.error_word, kernel="prefill"))
    torch.cuda.synchronize()
    manager.check_device_errors()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    err = np.abs(outs[1].float().cpu().numpy() - oracle_out(manager, batch, contiguous)).max()
    assert err <= 2e-2, err


def reference_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                        positions: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """The unfused path: nn.RMSNorm over head_dim, transpose, rope.py's half-split rotation."""
    x = torch.nn.functional.rms_norm(x, (x.shape[-1],), weight, eps).transpose(1, 2)  # [B, H, T, D]
    half = x.shape[-1] // 2
    c = cos[positions].unsqueeze(1)
    s = sin[positions].unsqueeze(1)
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * c + rotated * s).to(x.dtype)


@pytest.mark.parametrize("query_len", [1, 3, 130])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_fused_norm_rope_scatter_matches_unfused_path(query_len, dtype):
    lengths = [0, 127, 300]
    gen = torch.Generator(device="cuda").manual_seed(query_len)
    pages = sum(math.ceil((n + query_len) / 128) for n in lengths) + 2
    managers = []
    for _ in range(2):
        m = PagedKVCacheManager(2, 8, 128, pages * 128, 128, len(lengths), dtype, "cuda")
        W.shuffle_free_pages(m, 1)
        hs = [m.allocate() for _ in lengths]
        for h, n in zip(hs, lengths):
            m.reserve(h, n)
            h.length = n
        managers.append((m, hs))
    B, T = len(lengths), query_len
    q = torch.randn(B, T, 32, 128, generator=gen, device="cuda").to(dtype)
    k = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(dtype)
    v = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(dtype)
    wq = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    wk = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    cos, sin = W.rope_angles(torch.arange(8192, device="cuda"), 128)
    cos, sin = cos.contiguous(), sin.contiguous()
    positions = torch.tensor(lengths, device="cuda")[:, None] + torch.arange(T, device="cuda")[None, :]

    (m0, h0), (m1, h1) = managers
    b0 = m0.begin_batch(h0, T)
    q_ref = reference_norm_rope(q, wq, cos, sin, positions)
    k_ref = reference_norm_rope(k, wk, cos, sin, positions)
    b0.write_layer(1, k_ref, v.transpose(1, 2))
    b1 = m1.begin_batch(h1, T)
    q_fused = b1.prepare_layer(1, q, k, v, wq, wk, cos, sin)
    torch.cuda.synchronize()
    m1.check_device_errors()
    assert q_fused.shape == q_ref.shape
    assert (q_fused.float() - q_ref.float()).abs().max().item() <= 2e-2
    assert torch.equal(m0.v_cache, m1.v_cache)  # v is a byte copy
    assert (m0.k_cache.float() - m1.k_cache.float()).abs().max().item() <= 2e-2
    # same rounding steps as the unfused path: nearly every element agrees bit for bit
    same = (q_fused == q_ref).float().mean().item()
    assert same > 0.99, same
    # and attention over the fused writes equals attention over the unfused ones
    out0 = b0.attend_layer(q_ref, 1)
    out1 = b1.attend_layer(q_fused, 1)
    torch.cuda.synchronize()
    assert (out0.float() - out1.float()).abs().max().item() <= 2e-2


def test_fused_norm_rope_scatter_full_config3_chunk():
    """The fused kernel on config 3's whole chunk (8 requests x 512 tokens over prefixes
    U[0, 4096], shuffled pages): q against the unfused path, every written k/v row of the
    chunk read back out of its page slot (v bit for bit: a copy), no other pool row touched."""
    prefixes = [2998, 4045, 1590, 2020, 1436, 3762, 183, 2532]
    T, dtype = 512, torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(33)
    pages = sum(math.ceil((n + T) / 128) for n in prefixes) + 4
    m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(prefixes), dtype, "cuda")
    W.shuffle_free_pages(m, 33)
    hs = [m.allocate() for _ in prefixes]
    for h, n in zip(hs, prefixes):
        m.reserve(h, n)
        h.length = n
    B = len(prefixes)
    q = torch.randn(B, T, 32, 128, generator=gen, device="cuda").to(dtype)
    k = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(dtype)
    v = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(dtype)
    wq = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    wk = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    cos, sin = W.rope_angles(torch.arange(max(prefixes) + T, device="cuda"), 128)
    cos, sin = cos.contiguous(), sin.contiguous()
    positions = torch.tensor(prefixes, device="cuda")[:, None] + torch.arange(T, device="cuda")[None, :]
    m.k_cache.fill_(7.0)
    m.v_cache.fill_(7.0)
    batch = m.begin_batch(hs, T)
    q_fused = batch.prepare_layer(0, q, k, v, wq, wk, cos, sin)
    torch.cuda.synchronize()
    m.check_device_errors()
    q_ref = reference_norm_rope(q, wq, cos, sin, positions)
    k_ref = reference_norm_rope(k, wk, cos, sin, positions)
    assert (q_fused.float() - q_ref.float()).abs().max().item() <= 2e-2
    assert (q_fused == q_ref).float().mean().item() > 0.99
    # the chunk's rows, gathered from their page slots
    table = batch.page_table.long()
    slots = table.gather(1, positions // 128) * 128 + positions % 128  # [B, T]
    k_rows = m.k_cache[0, 0][:, slots]  # [H_kv, B, T, D]
    v_rows = m.v_cache[0, 0][:, slots]
    assert (k_rows.permute(1, 0, 2, 3).float() - k_ref.float()).abs().max().item() <= 2e-2
    assert torch.equal(v_rows.permute(1, 2, 0, 3), v)
    written = torch.zeros(m.k_cache.shape[3], dtype=torch.bool, device="cuda")
    written[slots.reshape(-1)] = True
    assert bool((m.k_cache[0, 0][:, ~written] == 7.0).all())
    assert bool((m.v_cache[0, 0][:, ~written] == 7.0).all())


@pytest.mark.parametrize("prefix, own, query_len", [(4096, 300, 1), (256, 1000, 1), (384, 130, 40)])
def test_shared_prefix_pages_attend_like_private_copies(prefix, own, query_len):
    """Requests aliasing a prefix's pages (share) attend exactly like requests holding copies."""
    gen = torch.Generator(device="cuda").manual_seed(prefix + own)
    n_req = 3
    pages = (math.ceil(prefix / 128) + math.ceil((own + query_len) / 128) + 1) * (n_req + 1) + 4
    outs = []
    for shared in (True, False):
        g = torch.Generator(device="cuda").manual_seed(prefix + own)
        m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, n_req + 1, torch.bfloat16, "cuda")
        W.shuffle_free_pages(m, 3)
        root = m.allocate()
        W.fill_history(m, root, prefix, g)
        handles = []
        for _ in range(n_req):
            if shared:
                h = m.share(root, prefix)
            else:
                h = m.allocate_for_request(m.snapshot(root))
            W.fill_history(m, h, prefix + own, g, start=prefix)
            handles.append(h)
        m.release(root)
        if shared:
            assert all(m.page_refcount(p) == n_req for p in handles[0].pages[:prefix // 128])
        q, k, v = W.step_inputs(m, handles, query_len, 32, g)
        batch = m.begin_batch(handles, query_len)
        batch.write_layer(0, k, v)
        outs.append(batch.attend_layer(q, 0).clone())
        torch.cuda.synchronize()
        m.check_device_errors()
    assert torch.equal(outs[0], outs[1])
