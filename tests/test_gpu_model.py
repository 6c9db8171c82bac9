"""Qwen3.5-hybrid harness against a plain fp32 PyTorch restatement of the
same model (a reduced configuration with the real head widths: 3 gated-DeltaNet
layers and 1 attention layer).

The reference below decodes every packed tensor bit-exactly (``decode``),
runs the model one token at a time in fp32 (dense projections, the
delta-rule recurrence written out per head, attention over the cache), and
is compared with the harness's prefill (tcgen05 matmul + torch attention),
its eager decode steps (fused matvec + the decode kernels) and its captured
CUDA-graph decode.  mlx_lm's model sources are not in the reference
repository, so the formulas are the ones written in include/gsq_model.h.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from gsq_b200.models import Qwen35Config, build_qwen35, random_weights
from gsq_b200.runtime.kernels import decode

pytestmark = pytest.mark.gpu

CFG = Qwen35Config(hidden_size=512, intermediate_size=768, num_hidden_layers=4, num_attention_heads=4,
                   num_key_value_heads=2, vocab_size=512, linear_num_value_heads=4, linear_num_key_heads=2)
TOL = 2e-2  # rel-L2 of logits: fp16 activations between projections + 16-bit activation quantisation


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


class Reference:
    """fp32, token by token."""

    def __init__(self, w, cfg, dev):
        self.cfg, self.w, self.dev = cfg, {}, dev
        for name, t in w.items():
            if hasattr(t, "quantization_type"):
                self.w[name] = decode(t.data, t.quantization_type).reshape(t.logical_shape).float()
            else:
                self.w[name] = t.float()
        c = cfg
        self.conv = {i: torch.zeros(3, c.gdn_conv_dim, device=dev) for i in range(c.num_hidden_layers)
                     if c.is_linear(i)}
        self.S = {i: torch.zeros(c.linear_num_value_heads, 128, 128, device=dev) for i in self.conv}
        self.K = {i: [] for i in range(c.num_hidden_layers) if not c.is_linear(i)}
        self.V = {i: [] for i in self.K}
        self.pos = 0

    @staticmethod
    def norm(x, w, eps):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * (w if w is not None else 1.0)

    def rope(self, x, pos):
        c = self.cfg
        rot = c.rotary_dim
        i = torch.arange(rot // 2, device=self.dev, dtype=torch.float64)
        ang = (pos * c.rope_theta ** (-2.0 * i / rot)).float()
        x1, x2 = x[..., :rot // 2], x[..., rot // 2:rot]
        return torch.cat([x1 * ang.cos() - x2 * ang.sin(), x2 * ang.cos() + x1 * ang.sin(), x[..., rot:]], -1)

    def step(self, tok):
        c, w, eps = self.cfg, self.w, self.cfg.rms_norm_eps
        x = w["token_embd.weight"][tok].clone()
        for i in range(c.num_hidden_layers):
            p = f"blk.{i}."
            h = self.norm(x, w[p + "attn_norm.weight"], eps)
            if c.is_linear(i):
                nk, nv = c.linear_num_key_heads, c.linear_num_value_heads
                qkv = w[p + "attn_qkv.weight"] @ h
                z = (w[p + "attn_gate.weight"] @ h).reshape(nv, 128)
                a = w[p + "ssm_alpha.weight"] @ h
                b = w[p + "ssm_beta.weight"] @ h
                win = torch.cat([self.conv[i], qkv[None]], 0)  # 4 x C, oldest first
                self.conv[i] = win[1:]
                cv = F.silu((win.T * w[p + "ssm_conv1d.weight"]).sum(-1))
                q = cv[:nk * 128].reshape(nk, 128)
                k = cv[nk * 128:2 * nk * 128].reshape(nk, 128)
                v = cv[2 * nk * 128:].reshape(nv, 128)
                q = self.norm(q, None, 1e-6) / 128.0
                k = self.norm(k, None, 1e-6) / math.sqrt(128.0)
                g = torch.exp(w[p + "ssm_a"] * F.softplus(a + w[p + "ssm_dt.bias"]))
                beta = torch.sigmoid(b)
                o = torch.empty(nv, 128, device=self.dev)
                for hh in range(nv):
                    kh = hh % nk
                    S = self.S[i][hh] * g[hh]             # [v index, k index]
                    u = (v[hh] - S @ k[kh]) * beta[hh]
                    S = S + u[:, None] * k[kh][None, :]
                    self.S[i][hh] = S
                    o[hh] = S @ q[kh]
                o = self.norm(o, w[p + "ssm_norm.weight"], eps) * F.silu(z)
                d = w[p + "ssm_out.weight"] @ o.reshape(-1)
            else:
                nq, nkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
                qg = (w[p + "attn_q.weight"] @ h).reshape(nq, 2 * hd)
                q, gate = qg[:, :hd], qg[:, hd:]
                k = (w[p + "attn_k.weight"] @ h).reshape(nkv, hd)
                v = (w[p + "attn_v.weight"] @ h).reshape(nkv, hd)
                q = self.rope(self.norm(q, w[p + "attn_q_norm.weight"], eps), self.pos)
                k = self.rope(self.norm(k, w[p + "attn_k_norm.weight"], eps), self.pos)
                self.K[i].append(k)
                self.V[i].append(v)
                Ks, Vs = torch.stack(self.K[i]), torch.stack(self.V[i])  # [t, nkv, hd]
                o = torch.empty(nq, hd, device=self.dev)
                for hh in range(nq):
                    kv = hh // (nq // nkv)
                    pr = torch.softmax(Ks[:, kv] @ q[hh] / math.sqrt(hd), 0)
                    o[hh] = (pr[:, None] * Vs[:, kv]).sum(0) * torch.sigmoid(gate[hh])
                d = w[p + "attn_output.weight"] @ o.reshape(-1)
            x = x + d
            h2 = self.norm(x, w[p + "post_attention_norm.weight"], eps)
            gu = F.silu(w[p + "ffn_gate.weight"] @ h2) * (w[p + "ffn_up.weight"] @ h2)
            x = x + w[p + "ffn_down.weight"] @ gu
        self.pos += 1
        return w["output.weight"] @ self.norm(x, w["output_norm.weight"], eps)


@pytest.fixture(scope="module")
def setup():
    dev = torch.device("cuda:0")
    w = random_weights(CFG, dev, seed=3)
    return dev, w


@pytest.mark.parametrize("T", [12, 3])  # tiled matmul prefill (rows >= 8) and the fused matvec (rows < 8)
def test_prefill_then_decode_matches_reference(setup, T):
    dev, w = setup
    model = build_qwen35(w, CFG, dev, max_len=64)
    ref = Reference(w, CFG, dev)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, CFG.vocab_size, (T,), generator=g)
    for t in prompt.tolist():
        rl = ref.step(t)
    logits = model.prefill(prompt.to(torch.int32).to(dev))
    e = rel(logits, rl)
    assert e <= TOL, f"prefill rel-L2 {e}"
    for t in torch.randint(0, CFG.vocab_size, (4,), generator=g).tolist():
        rl = ref.step(t)
        ml = model.decode_step(t)[0]
        e = rel(ml, rl)
        assert e <= TOL, f"decode rel-L2 {e}"
    torch.cuda.synchronize()


def test_graph_decode_matches_eager(setup):
    dev, w = setup
    prompt = torch.arange(9, dtype=torch.int32, device=dev) * 37 % CFG.vocab_size
    model = build_qwen35(w, CFG, dev, max_len=64)
    model.prefill(prompt)
    eager = [model.decode_step()[0].clone() for _ in range(5)]
    model.prefill(prompt)
    model.decode_step()
    model.capture_decode()
    for i in range(1, 5):
        model.replay_decode(1)
        e = rel(model.graph_logits[0], eager[i])
        assert e <= 1e-5, f"graph step {i}: rel {e}"
    assert model.n_pos == 9 + 5
    torch.cuda.synchronize()


@pytest.mark.parametrize("B", [3, 9])  # 3: the fused matvec with two-row tiles; 9: the tcgen05 matmul
def test_batched_decode_matches_single_sequences(setup, B):
    """fork(B) copies the prompt's state into B sequences; one batched decode
    step (batched gated-DeltaNet and attention kernels, projections over B
    rows) must give every sequence the logits a single-sequence model gives
    for the same tokens, over two steps."""
    dev, w = setup
    model = build_qwen35(w, CFG, dev, max_len=64, max_batch=B)
    one = build_qwen35(w, CFG, dev, max_len=64)
    prompt = torch.arange(7, dtype=torch.int32, device=dev) * 29 % CFG.vocab_size
    model.prefill(prompt)
    model.fork(B)
    toks = [(17 * b + 5) % CFG.vocab_size for b in range(B)]
    first = model.decode_step(toks).clone()
    nxt = first.argmax(-1).tolist()
    second = model.decode_step(nxt).clone()
    assert first.shape == (B, CFG.vocab_size)
    for b in range(B):
        one.prefill(prompt)
        e1 = rel(first[b], one.decode_step(toks[b])[0])
        e2 = rel(second[b], one.decode_step(nxt[b])[0])
        assert e1 <= TOL and e2 <= TOL, (b, e1, e2)
    torch.cuda.synchronize()
    from gsq_b200 import _lib
    assert _lib.device_status(dev) == 0


def test_batched_graph_decode_matches_eager(setup):
    dev, w = setup
    B = 8
    prompt = torch.arange(5, dtype=torch.int32, device=dev) * 11 % CFG.vocab_size
    toks = [(31 * b + 2) % CFG.vocab_size for b in range(B)]
    model = build_qwen35(w, CFG, dev, max_len=64, max_batch=B)
    model.prefill(prompt)
    model.fork(B)
    model.decode_step(toks)
    eager = [model.decode_step().clone() for _ in range(3)]
    model.prefill(prompt)
    model.fork(B)
    model.decode_step(toks)
    model.capture_decode()
    for i in range(3):
        model.replay_decode(1)
        e = rel(model.graph_logits, eager[i])
        assert e <= 1e-5, f"graph step {i}: rel {e}"
    torch.cuda.synchronize()


@pytest.mark.parametrize("qtype", ["IQ2_XS", "IQ2_S", "Q4_K", "IQ4_XS"])
@pytest.mark.parametrize("rows", [1, 3])
@pytest.mark.parametrize("n_out,k", [(1024, 5120), (256, 17408)])
def test_fused_swiglu_matvec(qtype, rows, n_out, k):
    """gsq_qmv_swiglu on an interleaved gate|up join against two separate
    matvecs and the SwiGLU product in fp32 (rows 1: one-row tiles; 3: two-row
    tiles; 17408 inputs: K split over CTAs)."""
    from gsq_b200.models.qwen35 import _Packed
    from gsq_b200.quant.synthetic import random_matrix_torch
    from gsq_b200.runtime import PackedWeight
    from gsq_b200.runtime.kernels import quantized_matvec
    dev = torch.device("cuda:0")
    g = random_matrix_torch(qtype, n_out, k, seed=11, device=dev)
    u = random_matrix_torch(qtype, n_out, k, seed=12, device=dev)
    pg = PackedWeight.from_packed("gate", g, qtype, (n_out, k), device=None)
    pu = PackedWeight.from_packed("up", u, qtype, (n_out, k), device=None)
    joined = _Packed([pg, pu], interleave=8)
    x = torch.randn(rows, k, device=dev, generator=torch.Generator(device=dev).manual_seed(2)).to(torch.float16)
    y = joined.swiglu(x, out_dtype=torch.float32)
    yg = quantized_matvec(x, g, qtype=qtype, out_features=n_out, in_features=k, out_dtype=torch.float32)
    yu = quantized_matvec(x, u, qtype=qtype, out_features=n_out, in_features=k, out_dtype=torch.float32)
    ref = F.silu(yg) * yu
    assert y.shape == (rows, n_out)
    assert rel(y, ref) <= 1e-5, rel(y, ref)
    # the matmul path (8 rows and more) on the same join, whose gate|up values
    # are rounded to fp16 (the type the tensor-parallel gather delivers), then
    # gsq_silu_mul with group 8 in fp32; the joined and the separate matmuls
    # may sum in different split orders, so a value can round to the
    # neighbouring fp16 number (2^-11 relative): bar 2e-4
    xm = torch.randn(12, k, device=dev, generator=torch.Generator(device=dev).manual_seed(3)).to(torch.float16)
    ym = joined.swiglu(xm, out_dtype=torch.float32)
    gm = quantized_matvec(xm, g, qtype=qtype, out_features=n_out, in_features=k, out_dtype=torch.float16)
    um = quantized_matvec(xm, u, qtype=qtype, out_features=n_out, in_features=k, out_dtype=torch.float16)
    refm = F.silu(gm.float()) * um.float()
    assert rel(ym, refm) <= 2e-4, rel(ym, refm)


@pytest.mark.parametrize("group,n", [(8, 1024), (0, 1024), (4, 1020), (0, 1020)])
@pytest.mark.parametrize("in_dt", [torch.float32, torch.float16, torch.bfloat16])
def test_silu_mul(group, n, in_dt):
    """gsq_silu_mul against torch in fp32 for each input type: interleaved
    (group 8, the eight-per-thread kernel; group 4, the per-value kernel) and
    halves layouts, with n a multiple of 8 and not."""
    from gsq_b200.models.qwen35 import silu_mul
    dev = torch.device("cuda:0")
    rows = 5
    gu = torch.randn(rows, 2 * n, device=dev, generator=torch.Generator(device=dev).manual_seed(n)).to(in_dt)
    f = gu.float()
    if group:
        v = f.reshape(rows, n // group, 2, group)
        g, u = v[:, :, 0].reshape(rows, n), v[:, :, 1].reshape(rows, n)
    else:
        g, u = f[:, :n], f[:, n:]
    ref = F.silu(g) * u
    for out_dt in (torch.float32, torch.float16):
        y = silu_mul(gu, out_dt, group=group)
        assert y.dtype == out_dt
        assert rel(y, ref) <= (1e-5 if out_dt == torch.float32 else 5e-4), (out_dt, rel(y, ref))


def test_model_from_gguf_and_container(setup, tmp_path):
    """The model's weights written as a GGUF checkpoint, read back (directly,
    and through the packed container) and built: the same logits as the model
    built from the weights in memory."""
    from gsq_b200.gguf import GGUFReader, convert_gguf_to_safetensors, write_model_gguf
    from gsq_b200.runtime import PackedModelStore
    dev, w = setup
    src = write_model_gguf(tmp_path / "tiny.gguf", w, {"general.architecture": "qwen35"})
    prompt = torch.arange(10, dtype=torch.int32, device=dev) * 13 % CFG.vocab_size
    ref = build_qwen35(w, CFG, dev, max_len=32).prefill(prompt)
    from_gguf = build_qwen35(GGUFReader(src).model_weights(dev), CFG, dev, max_len=32).prefill(prompt)
    assert torch.equal(from_gguf, ref)
    dst = convert_gguf_to_safetensors(src, tmp_path / "tiny.safetensors")
    from_store = build_qwen35(PackedModelStore(dst, device=dev).model_weights(), CFG, dev, max_len=32).prefill(prompt)
    assert torch.equal(from_store, ref)


@pytest.mark.parametrize("T", [64, 200])
def test_gdn_prompt_matches_token_by_token(T):
    """gsq_gdn over a T-token prompt (conv/gate kernel, the scan over 16-column
    blocks, the gated-norm kernel) against T one-token calls (the single
    kernel of a decode token) on the same inputs, at the model's head counts
    (16 key / 48 value heads): the same outputs, final state and conv window."""
    from gsq_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    nk, nv = 16, 48
    C = 2 * nk * 128 + nv * 128
    g = torch.Generator(device=dev).manual_seed(7)
    proj = torch.randn(T, C + nv * 128, device=dev, generator=g)
    ab = (torch.randn(T, 2 * nv, device=dev, generator=g) * 1.5).half()
    cw = torch.randn(C, 4, device=dev, generator=g) * 0.3
    A = -torch.exp(torch.rand(nv, device=dev, generator=g) * 2)
    dtb = torch.randn(nv, device=dev, generator=g) * 0.5
    nw = 1 + 0.05 * torch.randn(128, device=dev, generator=g)
    state0 = torch.randn(nv, 128, 128, device=dev, generator=g) * 0.05
    conv0 = torch.randn(4, C, device=dev, generator=g)

    def call(rows, state, conv, pos, out):
        need = lib.gsq_gdn_scratch_bytes(rows.shape[0], nk, nv)
        scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        _lib.check(lib.gsq_gdn(rows.data_ptr(), rows.stride(0), ab_rows(rows).data_ptr(), ab.stride(0), None, 0, None,
                               0, rows.shape[0], nk, nv, conv.data_ptr(), pos.data_ptr(), cw.data_ptr(), A.data_ptr(),
                               dtb.data_ptr(), nw.data_ptr(), 1e-6, state.data_ptr(),
                               scratch.data_ptr() if need else None, need, out.data_ptr(), 0, _lib.stream_ptr(dev)))

    row_of = {}

    def ab_rows(rows):
        return ab[row_of[rows.data_ptr()]:]

    s_all, c_all = state0.clone(), conv0.clone()
    out_all = torch.empty(T, nv * 128, device=dev)
    row_of[proj.data_ptr()] = 0
    call(proj, s_all, c_all, torch.zeros(1, dtype=torch.int32, device=dev), out_all)
    s_one, c_one = state0.clone(), conv0.clone()
    out_one = torch.empty(T, nv * 128, device=dev)
    pos = torch.zeros(1, dtype=torch.int32, device=dev)
    for t in range(T):
        row = proj[t:t + 1]
        row_of[row.data_ptr()] = t
        pos.fill_(t)
        call(row, s_one, c_one, pos, out_one[t:t + 1])
    torch.cuda.synchronize()
    assert lib.gsq_device_status(None) == 0
    assert rel(out_all, out_one) <= 1e-4, rel(out_all, out_one)
    assert rel(s_all, s_one) <= 1e-4, rel(s_all, s_one)
    assert torch.equal(c_all, c_one)
