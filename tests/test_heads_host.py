"""Head-split layouts (gsq_b200/parallel/heads.py) and the input-block split
(InputParallelLinear), on CPU.

Checked here:
  * the head plans partition the heads, keep the reference's cyclic
    gated-DeltaNet routing (value head h reads key head h % nk,
    mlx_gsq/models/qwen35.py:87-94) and the GQA grouping on every rank, and
    give each rank whole 256-wide input blocks of the output projection;
  * row and input-block selections of packed matrices are bit-exact (the C
    oracle's dequantization of the selection equals the same rows / columns
    of the whole matrix's), for all 11 types;
  * a layer computed head-split, each rank's partial output projection then
    summed, equals the whole layer (float64 restatements of the
    gated-DeltaNet block, of the gated attention block and of the SwiGLU
    FFN, with rel-L2 <= 1e-12);
  * the whole model (``head_split_weights``): a small Qwen3.5-hybrid model
    with random packed weights (dequantised by the C oracle), run in float64
    by 2 and 4 ranks' head-split weights in lockstep, gives the whole
    model's prompt logits (rel-L2 <= 1e-10);
  * InputParallelLinear on 2 and 4 gloo ranks: the reduced partials equal
    the whole product on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsq_b200.parallel import (attention_heads, block_bounds, ffn_blocks, linear_attention_heads,
                               take_input_blocks, take_rows)
from gsq_b200.quant.layouts import SUPPORTED_QUANT_TYPES
from gsq_b200.quant.synthetic import random_activations, random_matrix

F64_TOL = 1e-12


def _rel(a, e):
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-300))


# ---------------------------------------------------------------- head plans

@pytest.mark.parametrize("nk,nv,world", [(16, 48, 1), (16, 48, 2), (16, 48, 4), (16, 48, 8), (4, 12, 2)])
def test_linear_attention_plan(nk, nv, world):
    dk = dv = 128
    keys, values, blocks = [], [], []
    for r in range(world):
        p = linear_attention_heads(nk, nv, world, r)
        m = len(p.key_heads)
        # the cyclic routing holds on the local heads: local value j reads local key j % m
        for j, h in enumerate(p.value_heads):
            assert p.key_heads[j % m] == h % nk
        assert len(p.qkv_rows(dk, dv)) == 2 * m * dk + len(p.value_heads) * dv
        assert len(p.gate_rows(dv)) == len(p.value_heads) * dv
        keys += p.key_heads
        values += p.value_heads
        blocks += p.out_blocks(dv)
    assert sorted(keys) == list(range(nk))
    assert sorted(values) == list(range(nv))
    assert sorted(blocks) == list(range(nv * dv // 256))


def test_linear_attention_plan_rejects_partial_blocks():
    with pytest.raises(ValueError):
        linear_attention_heads(16, 48, 16, 0)  # one 128-wide value head per repeat: half a block
    with pytest.raises(ValueError):
        linear_attention_heads(16, 48, 3, 0)
    with pytest.raises(ValueError):
        linear_attention_heads(16, 40, 2, 0)
    with pytest.raises(ValueError):
        linear_attention_heads(16, 48, 2, 2)


@pytest.mark.parametrize("nq,nkv,world", [(24, 4, 1), (24, 4, 2), (24, 4, 4), (24, 4, 8), (8, 2, 8)])
def test_attention_plan(nq, nkv, world):
    hd, g = 256, nq // nkv
    queries, blocks = [], []
    for r in range(world):
        p = attention_heads(nq, nkv, world, r)
        m, mk = len(p.query_heads), len(p.kv_heads)
        assert m % mk == 0
        for j, h in enumerate(p.query_heads):  # the grouped rule on the local heads
            assert p.kv_heads[j // (m // mk)] == h // g
        assert len(p.q_rows(hd)) == 2 * m * hd and len(p.kv_rows(hd)) == mk * hd
        queries += p.query_heads
        blocks += p.out_blocks(hd)
    assert sorted(queries) == list(range(nq))
    assert sorted(blocks) == list(range(nq * hd // 256))
    with pytest.raises(ValueError):
        attention_heads(24, 4, 16, 0)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8])
def test_ffn_blocks_partition(world):
    runs = [ffn_blocks(17408, world, r) for r in range(world)]
    assert runs[0].start == 0 and runs[-1].stop == 68
    assert all(a.stop == b.start for a, b in zip(runs, runs[1:]))
    assert max(len(r) for r in runs) - min(len(r) for r in runs) <= 1
    assert block_bounds(17408, world, world - 1) == (runs[-1].start, runs[-1].stop)
    with pytest.raises(ValueError):
        ffn_blocks(17408 + 128, world, 0)


# ------------------------------------------------- packed selections (exact)

@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_take_rows_and_input_blocks_are_exact(qtype, oracle_mod):
    n, k = 24, 1024
    packed = random_matrix(qtype, n, k, seed=5)
    full = oracle_mod.dequantize_c(packed, qtype).reshape(n, k)
    t = torch.from_numpy(packed)
    rows = [5, 0, 23, 7, 7]
    sel = take_rows(t, qtype, n, k, rows).numpy()
    np.testing.assert_array_equal(oracle_mod.dequantize_c(sel, qtype).reshape(len(rows), k), full[rows])
    blocks = [3, 1]
    cols = [b * 256 + i for b in blocks for i in range(256)]
    sub = take_input_blocks(t, qtype, n, k, blocks).numpy()
    np.testing.assert_array_equal(oracle_mod.dequantize_c(sub, qtype).reshape(n, 512), full[:, cols])
    with pytest.raises(ValueError):
        take_rows(t, qtype, n, k, [n])
    with pytest.raises(ValueError):
        take_input_blocks(t, qtype, n, k, [4])
    with pytest.raises(ValueError):
        take_input_blocks(t[:-1], qtype, n, k, [0])


@pytest.mark.parametrize("qtype", ["Q4_K", "IQ2_XS", "IQ4_XS"])
@pytest.mark.parametrize("world", [2, 3])
def test_input_block_partials_sum_to_the_product(qtype, world, oracle_mod):
    n, k = 40, 1536
    packed = random_matrix(qtype, n, k, seed=8)
    x = random_activations(3, k, seed=2).astype(np.float32)
    full = oracle_mod.matmul_c(x, packed, qtype, n, k)
    acc = np.zeros_like(full, dtype=np.float64)
    for r in range(world):
        b0, b1 = block_bounds(k, world, r)
        sub = take_input_blocks(torch.from_numpy(packed), qtype, n, k, range(b0, b1)).numpy()
        acc += oracle_mod.matmul_c(np.ascontiguousarray(x[:, 256 * b0:256 * b1]), sub, qtype, n, 256 * (b1 - b0))
    assert _rel(acc, full) < 1e-5


# ------------------------------------ float64 layers: head split == whole

def _silu(x):
    return x / (1.0 + np.exp(-x))


def _rms(x, w=None, eps=1e-6):
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return y * w if w is not None else y


def _gdn(qkv, z, a, b, conv_w, ssm_a, dt_bias, norm_w, nk, nv, d=128):
    """The gated-DeltaNet block of one sequence from an empty state, float64:
    the reference's _gguf_gated_delta_call (mlx_gsq/models/qwen35.py:48-106)
    with mlx-lm's gated delta rule (conv + silu, unweighted q/k RMS norms
    scaled by 1/d and 1/sqrt(d), cyclic head routing, decay
    exp(-exp(A_log) * softplus(a + dt_bias)) with A_log = log(-ssm_a),
    write gate sigmoid(b), then RMS norm with weight times silu(z))."""
    T = qkv.shape[0]
    xin = np.concatenate([np.zeros((3, qkv.shape[1])), qkv], 0)
    c = _silu(np.stack([(xin[t:t + 4].T * conv_w).sum(-1) for t in range(T)]))
    q = d ** -1.0 * _rms(c[:, :nk * d].reshape(T, nk, d))
    k = d ** -0.5 * _rms(c[:, nk * d:2 * nk * d].reshape(T, nk, d))
    v = c[:, 2 * nk * d:].reshape(T, nv, d)
    beta = 1.0 / (1.0 + np.exp(-b))
    g = np.exp(-np.exp(np.log(-ssm_a)) * np.logaddexp(0.0, a + dt_bias))
    S = np.zeros((nv, d, d))
    out = np.empty((T, nv, d))
    for t in range(T):
        for h in range(nv):
            kh, qh = k[t, h % nk], q[t, h % nk]
            S[h] *= g[t, h]
            S[h] += np.outer((v[t, h] - S[h] @ kh) * beta[t, h], kh)
            out[t, h] = S[h] @ qh
    return (_rms(out, norm_w) * _silu(z.reshape(T, nv, d))).reshape(T, nv * d)


@pytest.mark.parametrize("nk,nv,world", [(4, 12, 2), (8, 24, 4)])
def test_gated_deltanet_head_split_sums_to_the_layer(nk, nv, world):
    rng = np.random.default_rng(3)
    d, T, H = 128, 5, 96
    C = 2 * nk * d + nv * d
    qkv = rng.normal(size=(T, C))
    z, a, b = rng.normal(size=(T, nv * d)), rng.normal(size=(T, nv)), rng.normal(size=(T, nv))
    conv_w = rng.normal(0.0, 0.5, (C, 4))
    ssm_a = -np.exp(rng.uniform(-1.5, 1.0, nv))
    dt_bias = rng.uniform(-1.0, 1.0, nv)
    norm_w = 1.0 + 0.1 * rng.normal(size=d)
    w_out = rng.normal(size=(H, nv * d)) / np.sqrt(nv * d)
    whole = _gdn(qkv, z, a, b, conv_w, ssm_a, dt_bias, norm_w, nk, nv) @ w_out.T
    acc = np.zeros_like(whole)
    for r in range(world):
        p = linear_attention_heads(nk, nv, world, r)
        rows, vh = p.qkv_rows(d, d), list(p.value_heads)
        loc = _gdn(qkv[:, rows], z[:, p.gate_rows(d)], a[:, vh], b[:, vh], conv_w[rows], ssm_a[vh], dt_bias[vh],
                   norm_w, len(p.key_heads), len(vh))
        cols = [blk * 256 + i for blk in p.out_blocks(d) for i in range(256)]
        acc += loc @ w_out[:, cols].T
    assert _rel(acc, whole) < F64_TOL


def _rope(x, pos, rot, theta):
    inv = theta ** (-np.arange(0, rot, 2) / rot)
    ang = pos[:, None] * inv[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2 = x[..., :rot // 2], x[..., rot // 2:rot]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin, x[..., rot:]], -1)


def _attention(p, nq, nkv, q_norm, k_norm, hd=256, rot=64, theta=1e7):
    """Gated GQA attention of a prompt from position 0, float64: per query
    head hd query values then hd gate values, weighted RMS norms of q and k,
    partial rotary embedding, causal softmax(q k^T / sqrt(hd)) v, times
    sigmoid(gate); query head h reads key/value head h // (nq/nkv)."""
    T = p.shape[0]
    qg = p[:, :nq * 2 * hd].reshape(T, nq, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:]
    k = p[:, nq * 2 * hd:nq * 2 * hd + nkv * hd].reshape(T, nkv, hd)
    v = p[:, nq * 2 * hd + nkv * hd:].reshape(T, nkv, hd)
    pos = np.arange(T, dtype=np.float64)
    q, k = _rope(_rms(q, q_norm), pos, rot, theta), _rope(_rms(k, k_norm), pos, rot, theta)
    out = np.empty((T, nq, hd))
    mask = np.triu(np.full((T, T), -np.inf), 1)
    for h in range(nq):
        kv = h // (nq // nkv)
        s = q[:, h] @ k[:, kv].T / np.sqrt(hd) + mask
        e = np.exp(s - s.max(-1, keepdims=True))
        out[:, h] = (e / e.sum(-1, keepdims=True)) @ v[:, kv]
    return (out / (1.0 + np.exp(-gate))).reshape(T, nq * hd)


@pytest.mark.parametrize("nq,nkv,world", [(8, 2, 2), (8, 2, 8), (12, 2, 4)])
def test_attention_head_split_sums_to_the_layer(nq, nkv, world):
    rng = np.random.default_rng(4)
    hd, T, H = 256, 6, 80
    pq = rng.normal(size=(T, 2 * nq * hd))
    pk, pv = rng.normal(size=(T, nkv * hd)), rng.normal(size=(T, nkv * hd))
    q_norm, k_norm = 1.0 + 0.1 * rng.normal(size=hd), 1.0 + 0.1 * rng.normal(size=hd)
    w_o = rng.normal(size=(H, nq * hd)) / np.sqrt(nq * hd)
    whole = _attention(np.concatenate([pq, pk, pv], 1), nq, nkv, q_norm, k_norm) @ w_o.T
    acc = np.zeros_like(whole)
    for r in range(world):
        p = attention_heads(nq, nkv, world, r)
        kvr = p.kv_rows(hd)
        loc = _attention(np.concatenate([pq[:, p.q_rows(hd)], pk[:, kvr], pv[:, kvr]], 1), len(p.query_heads),
                         len(p.kv_heads), q_norm, k_norm)
        cols = [blk * 256 + i for blk in p.out_blocks(hd) for i in range(256)]
        acc += loc @ w_o[:, cols].T
    assert _rel(acc, whole) < F64_TOL


@pytest.mark.parametrize("world", [2, 3])
def test_ffn_block_split_sums_to_the_layer(world):
    rng = np.random.default_rng(6)
    H, inter, T = 64, 1280, 4
    x = rng.normal(size=(T, H))
    wg, wu = rng.normal(size=(inter, H)), rng.normal(size=(inter, H))
    wd = rng.normal(size=(H, inter)) / np.sqrt(inter)
    whole = (_silu(x @ wg.T) * (x @ wu.T)) @ wd.T
    acc = np.zeros_like(whole)
    for r in range(world):
        blk = ffn_blocks(inter, world, r)
        sl = slice(256 * blk.start, 256 * blk.stop)
        acc += (_silu(x @ wg[sl].T) * (x @ wu[sl].T)) @ wd[:, sl].T
    assert _rel(acc, whole) < F64_TOL


# ---------------------------------------- InputParallelLinear on gloo ranks

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, qtype, result_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import oracle
    from gsq_b200.parallel import InputParallelLinear
    from gsq_b200.runtime import PackedWeight
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 32, 1280  # 5 input blocks: uneven over 2 and 4 ranks
        packed = random_matrix(qtype, n, k, seed=12)
        w = PackedWeight.from_packed("w", packed, qtype, (n, k), device=None)
        x = torch.from_numpy(random_activations(2, k, seed=3).astype(np.float32))
        holder = []

        def local(xx):
            s = holder[0]
            return torch.from_numpy(oracle.matmul_c(xx.numpy(), s.data.numpy(), qtype, n, s.logical_shape[1]))

        layer = InputParallelLinear(w, local_fn=local)
        holder.append(layer.shard)
        y = layer(layer.local_columns(x))
        exp = oracle.matmul_c(x.numpy(), packed, qtype, n, k)
        ok = y.shape == (2, n) and y.dtype == torch.float32 and np.allclose(y.numpy(), exp, rtol=1e-5, atol=1e-5)
        # every rank holds the same sum
        g = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(g, y)
        ok = ok and all(torch.equal(g[0], t) for t in g)
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_input_parallel_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, "Q4_K", q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = sorted(q.get(timeout=5) for _ in range(world))
    assert results == [(r, True) for r in range(world)]


# ------------------------- the whole model: head-split weights, float64

def _model64(rank_weights, rank_cfgs, ids, dense):
    """Prompt logits of the Qwen3.5-hybrid model from position 0, float64,
    run by every rank's weights in lockstep: each block's output projection
    (ssm_out, attn_output, ffn_down) is each rank's partial, summed over the
    ranks before the residual add; embedding, norms and LM head are whole.
    One rank with the whole weights is the whole model."""
    cfg0 = rank_cfgs[0]
    eps = cfg0.rms_norm_eps
    W0 = rank_weights[0]
    x = dense(W0["token_embd.weight"])[ids]
    for i in range(cfg0.num_hidden_layers):
        p = f"blk.{i}."
        h = _rms(x, W0[p + "attn_norm.weight"].double().numpy(), eps)
        d = 0.0
        for W, c in zip(rank_weights, rank_cfgs):
            if c.is_linear(i):
                nk, nv = c.linear_num_key_heads, c.linear_num_value_heads
                qkv, z = h @ dense(W[p + "attn_qkv.weight"]).T, h @ dense(W[p + "attn_gate.weight"]).T
                a = h @ W[p + "ssm_alpha.weight"].double().numpy().T
                b = h @ W[p + "ssm_beta.weight"].double().numpy().T
                o = _gdn(qkv, z, a, b, W[p + "ssm_conv1d.weight"].double().numpy(), W[p + "ssm_a"].double().numpy(),
                         W[p + "ssm_dt.bias"].double().numpy(), W[p + "ssm_norm.weight"].double().numpy(), nk, nv)
                d = d + o @ dense(W[p + "ssm_out.weight"]).T
            else:
                pr = np.concatenate([h @ dense(W[p + n]).T for n in ("attn_q.weight", "attn_k.weight",
                                                                     "attn_v.weight")], 1)
                o = _attention(pr, c.num_attention_heads, c.num_key_value_heads,
                               W[p + "attn_q_norm.weight"].double().numpy(),
                               W[p + "attn_k_norm.weight"].double().numpy(), hd=c.head_dim, rot=c.rotary_dim,
                               theta=c.rope_theta)
                d = d + o @ dense(W[p + "attn_output.weight"]).T
        x = x + d
        h2 = _rms(x, W0[p + "post_attention_norm.weight"].double().numpy(), eps)
        f = 0.0
        for W in rank_weights:
            g, u = h2 @ dense(W[p + "ffn_gate.weight"]).T, h2 @ dense(W[p + "ffn_up.weight"]).T
            f = f + (_silu(g) * u) @ dense(W[p + "ffn_down.weight"]).T
        x = x + f
    return _rms(x, W0["output_norm.weight"].double().numpy(), eps) @ dense(W0["output.weight"]).T


@pytest.mark.parametrize("world", [2, 4])
def test_head_split_weights_compute_the_whole_model(world, oracle_mod):
    from gsq_b200.models import Qwen35Config, head_split_weights, random_weights, tensor_shapes
    cfg = Qwen35Config(hidden_size=512, intermediate_size=1280, num_hidden_layers=4, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=320, linear_num_value_heads=24, linear_num_key_heads=8)
    weights = random_weights(cfg, "cpu", seed=1)
    cache = {}

    def dense(w):
        key = id(w)
        if key not in cache:
            n, k = w.logical_shape
            cache[key] = oracle_mod.dequantize_c(w.data.numpy(), w.quantization_type).reshape(n, k).astype(np.float64)
        return cache[key]

    ranks = [head_split_weights(weights, cfg, world, r) for r in range(world)]
    for w, c in ranks:  # every local tensor has the shape the local configuration names
        for name, shape in tensor_shapes(c).items():
            got = w[name].logical_shape if hasattr(w[name], "logical_shape") else tuple(w[name].shape)
            assert tuple(got) == tuple(shape), (name, got, shape)
    assert sum(c.intermediate_size for _, c in ranks) == cfg.intermediate_size
    assert sum(c.linear_num_value_heads for _, c in ranks) == cfg.linear_num_value_heads
    ids = np.array([3, 17, 250, 99, 3])
    whole = _model64([weights], [cfg], ids, dense)
    split = _model64([w for w, _ in ranks], [c for _, c in ranks], ids, dense)
    assert np.all(np.isfinite(whole))
    assert _rel(split, whole) < 1e-10
