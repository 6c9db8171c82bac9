"""Qwen3.5-hybrid decoder over packed GGUF weights (the model harness).

The reference attaches packed weights to mlx_lm's Qwen3.5 model
(``mlx_gsq/models/qwen35.py:11-152``): 64 decoder layers at hidden 5120,
every 4th layer gated GQA attention (24 query heads, 4 key/value heads of
256), the others gated-DeltaNet linear attention (16 key heads and 48 value
heads of 128, value head h reading key head h % 16, ``qwen35.py:87-94``),
SwiGLU FFN 17408, vocab 248320.  Here the same model runs on B200:

  * every quantized projection is a packed-weight kernel call
    (``quantized_matvec``: the fused dequant-matvec for fewer than 8 token
    rows, the tcgen05 dequant-matmul above), with fp16 activations in and
    fp32 out;
  * the projections of a layer that read the same input and share a quant
    type are joined row-wise at load time (attn_qkv|attn_gate,
    attn_q|attn_k|attn_v, and ffn_gate|ffn_up interleaved in groups of 8
    rows): a packed matrix is rows of whole blocks, so the join is a byte
    rearrangement and each layer makes fewer, larger calls;
  * the FFN's gate|up matvec ends in the SwiGLU product (``gsq_qmv_swiglu``:
    each 16-row tile holds 8 gate rows and their 8 up rows, so the epilogue
    pairs them in-lane) and writes the down projection's fp16 input;
  * the work between projections is in ``include/gsq_model.h``: residual
    add + RMSNorm, SiLU-mul, the gated-DeltaNet block (conv, norms, gates,
    recurrence, gated norm) and the single-token attention step; prefill
    attention uses torch's scaled-dot-product attention;
  * a decode step (embedding gather -> 64 layers -> LM head -> argmax ->
    next id) reads its token and position from device buffers, so it is
    captured once as a CUDA graph and replayed per token.

GGUF tensor names and the A_log convention follow ``qwen35.py:104-152``
(``ssm_a`` holds -exp(A_log), ``qwen35.py:43-45``).  mlx_lm's Qwen3.5 and
gated-delta sources are not part of the reference repository; the formulas
used are written in ``include/gsq_model.h``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import _lib
from ..parallel.tp import reduce_partials
from ..runtime.kernels import packed_embedding, quantized_matvec
from ..runtime.store import PackedWeight


@dataclass(frozen=True)
class Qwen35Config:
    """Model dimensions (``qwen35.py:11-36``)."""
    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_hidden_layers: int = 64
    num_attention_heads: int = 24
    num_key_value_heads: int = 4
    head_dim: int = 256
    vocab_size: int = 248320
    rms_norm_eps: float = 1e-6
    linear_num_value_heads: int = 48
    linear_num_key_heads: int = 16
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    full_attention_interval: int = 4
    rope_theta: float = 10_000_000.0
    partial_rotary_factor: float = 0.25

    def is_linear(self, i: int) -> bool:
        return (i + 1) % self.full_attention_interval != 0

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.linear_num_key_heads * self.linear_key_head_dim + \
            self.linear_num_value_heads * self.linear_value_head_dim

    def check(self) -> None:
        if self.linear_key_head_dim != 128 or self.linear_value_head_dim != 128 or self.head_dim != 256:
            raise ValueError("the harness kernels need 128-wide linear-attention heads and 256-wide attention heads")
        if self.linear_conv_kernel_dim != 4:
            raise ValueError("the conv kernel width must be 4")
        if self.linear_num_value_heads % self.linear_num_key_heads or \
                self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("head counts must divide")


def tensor_shapes(cfg: Qwen35Config) -> dict[str, tuple[int, ...]]:
    """Logical shapes (out, in) of every GGUF tensor of the model, by name."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    nq, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    nv, dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
    s = {"token_embd.weight": (cfg.vocab_size, H), "output_norm.weight": (H,), "output.weight": (cfg.vocab_size, H)}
    for i in range(cfg.num_hidden_layers):
        p = f"blk.{i}."
        s[p + "attn_norm.weight"] = (H,)
        s[p + "post_attention_norm.weight"] = (H,)
        s[p + "ffn_gate.weight"] = (I, H)
        s[p + "ffn_up.weight"] = (I, H)
        s[p + "ffn_down.weight"] = (H, I)
        if cfg.is_linear(i):
            s[p + "attn_qkv.weight"] = (cfg.gdn_conv_dim, H)
            s[p + "attn_gate.weight"] = (nv * dv, H)
            s[p + "ssm_out.weight"] = (H, nv * dv)
            s[p + "ssm_alpha.weight"] = (nv, H)
            s[p + "ssm_beta.weight"] = (nv, H)
            s[p + "ssm_conv1d.weight"] = (cfg.gdn_conv_dim, cfg.linear_conv_kernel_dim)
            s[p + "ssm_a"] = (nv,)
            s[p + "ssm_dt.bias"] = (nv,)
            s[p + "ssm_norm.weight"] = (dv,)
        else:
            s[p + "attn_q.weight"] = (2 * nq * hd, H)
            s[p + "attn_k.weight"] = (nkv * hd, H)
            s[p + "attn_v.weight"] = (nkv * hd, H)
            s[p + "attn_output.weight"] = (H, nq * hd)
            s[p + "attn_q_norm.weight"] = (hd,)
            s[p + "attn_k_norm.weight"] = (hd,)
    return s


def default_type_mix(cfg: Qwen35Config) -> dict[str, str]:
    """Quant type per packed tensor of the benchmarked 27B model: embedding
    and LM head Q6_K; FFN gate/up IQ2_XS on even layers, IQ2_S on odd ones; FFN down
    Q4_K; attention and linear-attention projections IQ3_S on even layers,
    IQ4_XS on odd ones.  ssm_alpha / ssm_beta, norms, conv taps and gates
    stay plain (F32)."""
    mix = {"token_embd.weight": "Q6_K", "output.weight": "Q6_K"}
    for i in range(cfg.num_hidden_layers):
        p = f"blk.{i}."
        mix[p + "ffn_gate.weight"] = mix[p + "ffn_up.weight"] = "IQ2_XS" if i % 2 == 0 else "IQ2_S"
        mix[p + "ffn_down.weight"] = "Q4_K"
        att = "IQ3_S" if i % 2 == 0 else "IQ4_XS"
        names = ("attn_qkv", "attn_gate", "ssm_out") if cfg.is_linear(i) else \
            ("attn_q", "attn_k", "attn_v", "attn_output")
        for n in names:
            mix[p + n + ".weight"] = att
    return mix


def random_weights(cfg: Qwen35Config, device, seed: int = 0, type_mix: dict[str, str] | None = None) -> dict:
    """Random-init weights of the model by GGUF name, on ``device``: packed
    tensors as ``PackedWeight`` (the synthetic generator of the benchmarks:
    uniform bytes, fp16 super-block scales in [1e-4, 4e-3]), plain tensors as
    fp32 (norm weights near 1, conv taps, gates)."""
    from ..quant.synthetic import random_matrix_torch
    cfg.check()
    mix = type_mix or default_type_mix(cfg)
    gen = torch.Generator(device=device).manual_seed(seed)

    def rnd(shape, scale, offset=0.0):
        return torch.randn(shape, device=device, generator=gen) * scale + offset

    out = {}
    for idx, (name, shape) in enumerate(tensor_shapes(cfg).items()):
        if name in mix:
            data = random_matrix_torch(mix[name], shape[0], shape[1], seed=seed * 100003 + idx, device=device)
            out[name] = PackedWeight.from_packed(name, data, mix[name], shape, device=None)
        elif name.endswith("norm.weight"):
            out[name] = rnd(shape, 0.05, 1.0)
        elif name.endswith("ssm_conv1d.weight"):
            out[name] = rnd(shape, 0.3)
        elif name.endswith("ssm_alpha.weight") or name.endswith("ssm_beta.weight"):
            out[name] = rnd(shape, 1.0 / math.sqrt(shape[1]))
        elif name.endswith("ssm_a"):
            out[name] = -torch.exp(torch.rand(shape, device=device, generator=gen) * 2.0)
        elif name.endswith("ssm_dt.bias"):
            out[name] = rnd(shape, 0.5)
        else:
            raise KeyError(name)
    return out


def head_split_weights(weights: dict, cfg: Qwen35Config, world: int, rank: int) -> tuple[dict, Qwen35Config]:
    """One rank's weights of the head-split layout (``parallel/heads.py``),
    by GGUF name, and the rank's local configuration.

    Each gated-DeltaNet layer keeps the rank's key heads and the value heads
    that read them (``linear_attention_heads``). That covers its rows of
    attn_qkv, attn_gate, ssm_alpha, ssm_beta and the conv taps, its entries
    of ssm_a and ssm_dt.bias, and its input blocks of ssm_out. Each
    attention layer keeps its query heads and their key/value heads
    (``attention_heads``): its rows of attn_q, attn_k and attn_v, and its
    input blocks of attn_output. Each FFN keeps a run of 256-wide blocks of
    the intermediate width (``ffn_blocks``): those rows of ffn_gate and
    ffn_up, and the same input blocks of ffn_down. Embedding, LM head and
    norm weights are kept whole. Packed tensors are byte selections of the
    payload (``take_rows`` / ``take_input_blocks``), on the payload's
    device.

    The local configuration has the rank's head counts and intermediate
    width. Running the model on it, with the ranks' partial outputs of
    ssm_out, attn_output and ffn_down summed before each residual add,
    computes the whole model."""
    from dataclasses import replace
    from ..parallel.heads import attention_heads, ffn_blocks, linear_attention_heads, take_input_blocks, take_rows
    cfg.check()
    dk, dv, hd = cfg.linear_key_head_dim, cfg.linear_value_head_dim, cfg.head_dim
    gdn = linear_attention_heads(cfg.linear_num_key_heads, cfg.linear_num_value_heads, world, rank, dv)
    att = attention_heads(cfg.num_attention_heads, cfg.num_key_value_heads, world, rank, hd)
    ffn = ffn_blocks(cfg.intermediate_size, world, rank)
    inter = 256 * len(ffn)
    local = replace(cfg, linear_num_key_heads=len(gdn.key_heads), linear_num_value_heads=len(gdn.value_heads),
                    num_attention_heads=len(att.query_heads), num_key_value_heads=len(att.kv_heads),
                    intermediate_size=inter)

    def rows(name, idx):
        w = weights[name]
        n, k = w.logical_shape
        data = take_rows(w.data, w.quantization_type, n, k, idx)
        return PackedWeight.from_packed(f"{name}[rank {rank}/{world}]", data, w.quantization_type, (len(idx), k),
                                        device=None)

    def cols(name, blocks):
        w = weights[name]
        n, k = w.logical_shape
        data = take_input_blocks(w.data, w.quantization_type, n, k, blocks)
        return PackedWeight.from_packed(f"{name}[rank {rank}/{world}]", data, w.quantization_type,
                                        (n, 256 * len(blocks)), device=None)

    def plain(name, idx):
        t = weights[name]
        return t.index_select(0, torch.as_tensor(idx, dtype=torch.long, device=t.device)).contiguous()

    ffn_rows = list(range(256 * ffn.start, 256 * ffn.stop))
    out = {}
    for name in ("token_embd.weight", "output_norm.weight", "output.weight"):
        out[name] = weights[name]
    for i in range(cfg.num_hidden_layers):
        p = f"blk.{i}."
        for n in ("attn_norm.weight", "post_attention_norm.weight"):
            out[p + n] = weights[p + n]
        out[p + "ffn_gate.weight"] = rows(p + "ffn_gate.weight", ffn_rows)
        out[p + "ffn_up.weight"] = rows(p + "ffn_up.weight", ffn_rows)
        out[p + "ffn_down.weight"] = cols(p + "ffn_down.weight", list(ffn))
        if cfg.is_linear(i):
            qkv = gdn.qkv_rows(dk, dv)
            vh = list(gdn.value_heads)
            out[p + "attn_qkv.weight"] = rows(p + "attn_qkv.weight", qkv)
            out[p + "attn_gate.weight"] = rows(p + "attn_gate.weight", gdn.gate_rows(dv))
            out[p + "ssm_out.weight"] = cols(p + "ssm_out.weight", gdn.out_blocks(dv))
            out[p + "ssm_alpha.weight"] = plain(p + "ssm_alpha.weight", vh)
            out[p + "ssm_beta.weight"] = plain(p + "ssm_beta.weight", vh)
            conv = weights[p + "ssm_conv1d.weight"].reshape(-1, cfg.linear_conv_kernel_dim)  # [channel, tap]
            out[p + "ssm_conv1d.weight"] = conv.index_select(
                0, torch.as_tensor(qkv, dtype=torch.long, device=conv.device)).contiguous()
            out[p + "ssm_a"] = plain(p + "ssm_a", vh)
            out[p + "ssm_dt.bias"] = plain(p + "ssm_dt.bias", vh)
            out[p + "ssm_norm.weight"] = weights[p + "ssm_norm.weight"]
        else:
            kv = att.kv_rows(hd)
            out[p + "attn_q.weight"] = rows(p + "attn_q.weight", att.q_rows(hd))
            out[p + "attn_k.weight"] = rows(p + "attn_k.weight", kv)
            out[p + "attn_v.weight"] = rows(p + "attn_v.weight", kv)
            out[p + "attn_output.weight"] = cols(p + "attn_output.weight", att.out_blocks(hd))
            out[p + "attn_q_norm.weight"] = weights[p + "attn_q_norm.weight"]
            out[p + "attn_k_norm.weight"] = weights[p + "attn_k_norm.weight"]
    return out, local


class _Packed:
    """A packed projection: flat uint8 payload of n rows x k inputs.

    Several same-type projections of one input are joined row-wise; with
    ``interleave=g`` two of them (gate, up) alternate in groups of g rows
    (g gate rows, then the same g up rows), the layout of the fused SwiGLU
    matvec (``gsq_qmv_swiglu``)."""

    def __init__(self, parts: list[PackedWeight], interleave: int = 0):
        q = {p.quantization_type for p in parts}
        k = {p.logical_shape[1] for p in parts}
        if len(q) != 1 or len(k) != 1:
            raise ValueError("joined projections must share quant type and input width: "
                             + ", ".join(p.name for p in parts))
        self.qtype, self.k = q.pop(), k.pop()
        self.n = sum(p.logical_shape[0] for p in parts)
        self.interleave = interleave
        if interleave:
            if len(parts) != 2 or parts[0].logical_shape != parts[1].logical_shape or \
                    parts[0].logical_shape[0] % interleave:
                raise ValueError("interleaving needs two projections of equal shape, rows a multiple of the group")
            rb = parts[0].num_bytes // parts[0].logical_shape[0]
            g = [p.data.reshape(-1, interleave, rb) for p in parts]
            self.data = torch.stack(g, dim=1).reshape(-1)
        else:
            self.data = parts[0].data if len(parts) == 1 else torch.cat([p.data.reshape(-1) for p in parts])
        self.nbytes = self.data.numel()  # the whole projection's payload (all ranks together)
        self.world, self.rank, self.group, self.region = 1, 0, None, None
        self.prefill_region = None  # shared by the projections of the same width (tensor parallel)
        self.n_local, self.row0 = self.n, 0

    def shard(self, group) -> None:
        """Keep this rank's rows [r*n/P, (r+1)*n/P) (a byte slice of the
        payload) and create the call site's gather region (collective: every
        rank shards the same projections in the same order)."""
        from ..parallel import GatherRegion, shard_bounds
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        lo, hi = shard_bounds(self.n, world, rank)
        if self.interleave and lo % (2 * self.interleave):
            raise ValueError("a rank's rows must hold whole gate|up groups")
        rb = self.nbytes // self.n
        self.data = self.data[lo * rb:hi * rb].clone()
        self.world, self.rank, self.group = world, rank, group
        self.n_local, self.row0 = hi - lo, lo
        self.region = GatherRegion(1, self.n, group=group, device=self.data.device)

    def close(self) -> None:
        if self.region is not None:
            self.region.close()
            self.region = None

    def __call__(self, x16: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
        """x16 @ W.T as fp32 rows (``out_dtype`` fp16: rounded once from the
        fp32 sums, for prompts of 8 tokens and more; the tensor-parallel
        prompt path then returns the type of the projection's region)."""
        if self.world == 1:
            return quantized_matvec(x16, self.data, qtype=self.qtype, out_features=self.n, in_features=self.k,
                                    out_dtype=out_dtype)
        if x16.shape[0] == 1:  # decode: the gather is fused into the matvec (every rank's rows, over NVLink)
            from ..parallel import quantized_matvec_gather
            return quantized_matvec_gather(x16, self.data, qtype=self.qtype, out_features=self.n_local,
                                           in_features=self.k, region=self.region, row0=self.row0)
        reg = self.prefill_region
        if reg is not None and 8 <= x16.shape[0] <= reg.rows:  # prompt: the gather fused into the matmul epilogue
            from ..parallel import quantized_matmul_gather
            return quantized_matmul_gather(x16, self.data, qtype=self.qtype, out_features=self.n_local,
                                           in_features=self.k, region=reg, row0=self.row0)
        from ..parallel import gather_rows
        y = quantized_matvec(x16, self.data, qtype=self.qtype, out_features=self.n_local, in_features=self.k,
                             out_dtype=out_dtype)
        return gather_rows(y, self.group)

    def swiglu(self, x16: torch.Tensor, out_dtype=torch.float16) -> torch.Tensor:
        """silu(gate . x) * (up . x) of an interleaved gate|up join: one fused
        matvec below 8 rows, else the matmul then ``gsq_silu_mul``."""
        if self.interleave != 8:
            raise ValueError("swiglu needs the gate|up join interleaved in groups of 8")
        rows = x16.shape[0]
        if rows >= 8 or self.world > 1:
            # prompts: the gate|up values as fp16 (also what the gathered
            # tensor-parallel matmul delivers), then the SwiGLU kernel in fp32
            gu = self(x16, out_dtype=torch.float16 if rows >= 8 else torch.float32)
            return silu_mul(gu, out_dtype, group=8)
        from ..quant.layouts import type_id
        dev = x16.device
        lib = _lib.load()
        tid = type_id(self.qtype)
        need = lib.gsq_qmv_workspace_size(tid, self.n, self.k, rows)
        ws = _lib.workspaces.get(dev, need, "qmv")
        out = torch.empty((rows, self.n // 2), dtype=out_dtype, device=dev)
        _lib.check(lib.gsq_qmv_swiglu(tid, x16.data_ptr(), _lib.DTYPE_CODES[x16.dtype], self.data.data_ptr(),
                                      self.n // 2, self.k, rows, out.data_ptr(), _lib.DTYPE_CODES[out_dtype],
                                      ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                                      _stream(dev)))
        return out


def _stream(dev):
    return _lib.stream_ptr(dev)


def rmsnorm(resid: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float,
            out_dtype=torch.float16) -> torch.Tensor:
    """resid += delta (in place, when given); returns rmsnorm(resid) * weight."""
    rows, dim = resid.shape
    out = torch.empty((rows, dim), dtype=out_dtype, device=resid.device)
    _lib.check(_lib.load().gsq_rmsnorm(resid.data_ptr(), delta.data_ptr() if delta is not None else None, rows, dim,
                                       weight.data_ptr(), eps, out.data_ptr(), _lib.DTYPE_CODES[out_dtype],
                                       _stream(resid.device)))
    return out


def silu_mul(gu: torch.Tensor, out_dtype=torch.float16, group: int = 0) -> torch.Tensor:
    rows, n2 = gu.shape
    if gu.stride(1) != 1 or gu.stride(0) != n2:
        gu = gu.contiguous()
    out = torch.empty((rows, n2 // 2), dtype=out_dtype, device=gu.device)
    _lib.check(_lib.load().gsq_silu_mul(gu.data_ptr(), _lib.DTYPE_CODES[gu.dtype], rows, n2 // 2, group,
                                        out.data_ptr(), _lib.DTYPE_CODES[out_dtype], _stream(gu.device)))
    return out


class Qwen35:
    """The model, built from GGUF-named weights (``build_qwen35``).

    With ``group`` (an initialised process group of P ranks, one GPU each;
    tensor parallel) every packed projection is split by output rows over
    the ranks: decode tokens gather the rows inside the matvec kernel
    (``gsq_qmv_gather``), prompts inside the matmul epilogue
    (``gsq_qmm_gather``; prompts of 2-7 tokens, an NCCL all-gather).
    Norms, the gated-DeltaNet and attention blocks run on every rank on the
    gathered (identical) vectors.

    With ``reduce_group`` instead (the head-split layout,
    ``build_qwen35_head_split``) the weights and ``cfg`` are one rank's
    (``head_split_weights``): the blocks run on the rank's heads and
    intermediate blocks, the partial outputs of ssm_out / attn_output /
    ffn_down are summed over the ranks (NCCL all-reduce) before each
    residual add, and the LM head is split by vocabulary rows and gathered
    as with ``group``."""

    def __init__(self, weights: dict, cfg: Qwen35Config, device, max_len: int = 2304, group=None,
                 max_batch: int = 1, reduce_group=None):
        cfg.check()
        if max_batch < 1:
            raise ValueError("max_batch must be at least 1")
        if group is not None and reduce_group is not None:
            raise ValueError("a model splits by output rows (group) or by heads (reduce_group), not both")
        self.cfg, self.dev, self.max_len = cfg, torch.device(device), max_len
        self.max_batch, self.batch = int(max_batch), 1
        self.eps = cfg.rms_norm_eps
        w = weights
        self.embed = w["token_embd.weight"]
        self.out_norm = w["output_norm.weight"].float().contiguous()
        self.lm_head = _Packed([w["output.weight"]])
        nv = cfg.linear_num_value_heads
        nkv, hd = cfg.num_key_value_heads, cfg.head_dim
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"blk.{i}."
            L = {"linear": cfg.is_linear(i),
                 "attn_norm": w[p + "attn_norm.weight"].float().contiguous(),
                 "post_norm": w[p + "post_attention_norm.weight"].float().contiguous(),
                 "gate_up": _Packed([w[p + "ffn_gate.weight"], w[p + "ffn_up.weight"]], interleave=8),
                 "down": _Packed([w[p + "ffn_down.weight"]])}
            if L["linear"]:
                L["qkvz"] = _Packed([w[p + "attn_qkv.weight"], w[p + "attn_gate.weight"]])
                L["out"] = _Packed([w[p + "ssm_out.weight"]])
                L["ab"] = torch.cat([w[p + "ssm_alpha.weight"], w[p + "ssm_beta.weight"]]).to(torch.float16)
                L["conv_w"] = w[p + "ssm_conv1d.weight"].float().reshape(cfg.gdn_conv_dim, 4).contiguous()
                L["A"] = w[p + "ssm_a"].float().contiguous()
                L["dt_bias"] = w[p + "ssm_dt.bias"].float().contiguous()
                L["norm"] = w[p + "ssm_norm.weight"].float().contiguous()
                # per sequence of the batch: conv ring (slot = position & 3) and recurrent state
                L["conv_state"] = torch.zeros(max_batch, 4, cfg.gdn_conv_dim, device=self.dev)
                L["state"] = torch.zeros(max_batch, nv, cfg.linear_value_head_dim, cfg.linear_key_head_dim,
                                         device=self.dev)
            else:
                L["qkv"] = _Packed([w[p + "attn_q.weight"], w[p + "attn_k.weight"], w[p + "attn_v.weight"]])
                L["o"] = _Packed([w[p + "attn_output.weight"]])
                L["q_norm"] = w[p + "attn_q_norm.weight"].float().contiguous()
                L["k_norm"] = w[p + "attn_k_norm.weight"].float().contiguous()
                L["k_cache"] = torch.zeros(max_batch, max_len, nkv, hd, device=self.dev)
                L["v_cache"] = torch.zeros(max_batch, max_len, nkv, hd, device=self.dev)
            self.layers.append(L)
        self.world = dist.get_world_size(group) if group is not None else 1
        self.reduce_group = reduce_group if reduce_group is not None and dist.get_world_size(reduce_group) > 1 \
            else None
        if self.reduce_group is not None:
            self.lm_head.shard(self.reduce_group)  # vocabulary rows, gathered in the matvec (or by NCCL)
        self._prefill_regions = {}
        if self.world > 1:
            for pk in self._projections():
                pk.shard(group)
            # Prompts gather inside the matmul epilogue into one region per
            # output width and value type, shared by every projection of that
            # kind (the LM head only ever sees one row).  Sharing is safe
            # because two calls on a region always have another gathered call
            # between them: no rank finishes that call before every rank's
            # matmul has started storing, which each does only after the
            # kernel that consumed the previous output of the region has
            # completed.  The FFN's gate|up outputs (the widest, read only by
            # the SwiGLU kernel, which computes in fp32 from any input type)
            # gather as fp16: half the NVLink bytes of the largest gather;
            # every other projection's output stays fp32 (a gate|up width may
            # equal another projection's, so the type is part of the key).
            from ..parallel import GatherRegion

            def kind(pk):
                fp16 = any(pk is L["gate_up"] for L in self.layers)
                return pk.n, torch.float16 if fp16 else torch.float32

            for key in sorted({kind(pk) for pk in self._projections() if pk is not self.lm_head}, key=str):
                self._prefill_regions[key] = GatherRegion(max_len, key[0], group=group, device=self.dev,
                                                          dtype=key[1])
            for pk in self._projections():
                if pk is not self.lm_head:
                    pk.prefill_region = self._prefill_regions[kind(pk)]
        self.pos = torch.zeros(1, dtype=torch.int32, device=self.dev)   # next position (decode)
        self.cur_id = torch.zeros(max_batch, dtype=torch.int32, device=self.dev)  # tokens to feed next (decode)
        self.n_pos = 0  # host copy of the position (prefill bookkeeping)
        self._graph = None
        inv = cfg.rope_theta ** (-torch.arange(0, cfg.rotary_dim, 2, dtype=torch.float32) / cfg.rotary_dim)
        self._inv_freq = inv.to(self.dev)

    def _projections(self) -> list:
        """Every packed projection, in a fixed order (the same on all ranks)."""
        out = [self.lm_head]
        for L in self.layers:
            out += [L[key] for key in ("qkvz", "out", "qkv", "o", "gate_up", "down") if key in L]
        return out

    def close(self) -> None:
        """Release the gather regions (collective with ``group``)."""
        self._graph = None
        for pk in self._projections():
            pk.close()
            pk.prefill_region = None
        for reg in self._prefill_regions.values():
            reg.close()
        self._prefill_regions = {}

    # ---- sizes ----
    def packed_bytes_per_token(self) -> int:
        """Packed weight bytes one decode token reads over all ranks (every
        projection and the LM head; one embedding row)."""
        return sum(pk.nbytes for pk in self._projections()) + self.embed.num_bytes // self.cfg.vocab_size

    def reset(self) -> None:
        """Empties sequence 0 and makes it the only one (batch 1)."""
        for L in self.layers:
            if L["linear"]:
                L["conv_state"][0].zero_()
                L["state"][0].zero_()
        self.pos.zero_()
        self.n_pos = 0
        self.batch = 1
        self._graph = None

    def fork(self, batch: int) -> None:
        """Batched decode from the current state: sequences 1..batch-1 become
        copies of sequence 0 (conv rings, recurrent states, caches up to the
        current position, next token); decode steps then advance all of them
        together, one token per sequence."""
        if not 1 <= batch <= self.max_batch:
            raise ValueError(f"batch must be in 1..{self.max_batch}")
        n = self.n_pos
        for L in self.layers:
            if L["linear"]:
                L["conv_state"][1:batch].copy_(L["conv_state"][0:1].expand(batch - 1, -1, -1))
                L["state"][1:batch].copy_(L["state"][0:1].expand(batch - 1, -1, -1, -1))
            else:
                for key in ("k_cache", "v_cache"):
                    L[key][1:batch, :n].copy_(L[key][0:1, :n].expand(batch - 1, -1, -1, -1))
        self.cur_id[1:batch].copy_(self.cur_id[0:1].expand(batch - 1))
        self.batch = batch
        self._graph = None

    # ---- blocks ----
    def _gdn(self, L, p: torch.Tensor, h: torch.Tensor, decode: bool = False) -> torch.Tensor:
        """The gated-DeltaNet block on the q|k|v|z projection p of input h:
        a prompt of p.shape[0] tokens of sequence 0, or (``decode``) one token
        of each of the batch's p.shape[0] sequences.  The 2 x 48 gate rows
        (plain fp16) are a cuBLAS GEMM for prompts and for decode batches of 8
        sequences and more, and are computed inside the block's kernel for
        smaller decode batches (there every CTA of a head recomputes them, a
        cost that grows with the batch)."""
        cfg, T = self.cfg, p.shape[0]
        nk, nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        lib = _lib.load()
        if decode:
            out = torch.empty(T, nv * cfg.linear_value_head_dim, dtype=torch.float16, device=self.dev)
            ab = F.linear(h, L["ab"]) if T >= 8 else None
            _lib.check(lib.gsq_gdn_batch(p.data_ptr(), p.stride(0), ab.data_ptr() if ab is not None else None,
                                         ab.stride(0) if ab is not None else 0, h.data_ptr(), h.stride(0),
                                         L["ab"].data_ptr(), cfg.hidden_size, T, nk, nv, L["conv_state"].data_ptr(),
                                         self.pos.data_ptr(), L["conv_w"].data_ptr(), L["A"].data_ptr(),
                                         L["dt_bias"].data_ptr(), L["norm"].data_ptr(), self.eps,
                                         L["state"].data_ptr(), out.data_ptr(), _lib.DTYPE_CODES[torch.float16],
                                         _stream(self.dev)))
            return out
        need = lib.gsq_gdn_scratch_bytes(T, nk, nv)
        scratch = torch.empty(need, dtype=torch.uint8, device=self.dev) if need else None
        out = torch.empty(T, nv * cfg.linear_value_head_dim, dtype=torch.float16, device=self.dev)
        ab = F.linear(h, L["ab"]) if T >= 8 else None
        _lib.check(lib.gsq_gdn(p.data_ptr(), p.stride(0), ab.data_ptr() if ab is not None else None,
                               ab.stride(0) if ab is not None else 0, h.data_ptr(), h.stride(0), L["ab"].data_ptr(),
                               cfg.hidden_size, T, nk, nv, L["conv_state"].data_ptr(), self.pos.data_ptr(),
                               L["conv_w"].data_ptr(), L["A"].data_ptr(), L["dt_bias"].data_ptr(),
                               L["norm"].data_ptr(), self.eps, L["state"].data_ptr(),
                               scratch.data_ptr() if scratch is not None else None, need, out.data_ptr(),
                               _lib.DTYPE_CODES[torch.float16],
                               _stream(self.dev)))
        return out

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        rot = self.cfg.rotary_dim
        ang = pos.float()[:, None] * self._inv_freq[None, :]
        cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        x1, x2 = x[..., :rot // 2], x[..., rot // 2:rot]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, x[..., rot:]], dim=-1)

    def _attn_prefill(self, L, p: torch.Tensor, pos0: int) -> torch.Tensor:
        cfg, T = self.cfg, p.shape[0]
        nq, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        if pos0 != 0:
            raise NotImplementedError("multi-token calls start at position 0 (prefill of an empty cache)")
        qg = p[:, :nq * 2 * hd].reshape(T, nq, 2 * hd)
        q, gate = qg[..., :hd], qg[..., hd:]
        k = p[:, nq * 2 * hd:nq * 2 * hd + nkv * hd].reshape(T, nkv, hd)
        v = p[:, nq * 2 * hd + nkv * hd:].reshape(T, nkv, hd)
        q = F.rms_norm(q, (hd,), L["q_norm"], self.eps)
        k = F.rms_norm(k, (hd,), L["k_norm"], self.eps)
        pos = torch.arange(pos0, pos0 + T, device=self.dev)
        q, k = self._rope(q, pos), self._rope(k, pos)
        L["k_cache"][0, pos0:pos0 + T] = k
        L["v_cache"][0, pos0:pos0 + T] = v
        att = F.scaled_dot_product_attention(q.transpose(0, 1)[None].to(torch.float16),
                                             k.transpose(0, 1)[None].to(torch.float16),
                                             v.transpose(0, 1)[None].to(torch.float16), is_causal=True,
                                             enable_gqa=True, scale=1.0 / math.sqrt(hd))
        o = att[0].transpose(0, 1).float() * torch.sigmoid(gate)
        return o.reshape(T, nq * hd).to(torch.float16)

    def _attn_decode(self, L, p: torch.Tensor) -> torch.Tensor:
        """One decode token of each of the batch's p.shape[0] sequences."""
        cfg, B = self.cfg, p.shape[0]
        nq, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        out = torch.empty(B, nq * hd, dtype=torch.float16, device=self.dev)
        _lib.check(_lib.load().gsq_attn_decode_batch(p.data_ptr(), nq, nkv, L["q_norm"].data_ptr(),
                                                     L["k_norm"].data_ptr(), self.eps, cfg.rotary_dim,
                                                     cfg.rope_theta, L["k_cache"].data_ptr(),
                                                     L["v_cache"].data_ptr(), self.max_len, self.pos.data_ptr(),
                                                     out.data_ptr(), _lib.DTYPE_CODES[torch.float16], B,
                                                     _stream(self.dev)))
        return out

    def _layers(self, x: torch.Tensor, pos0: int | None) -> torch.Tensor:
        """Runs every layer over x (fp32 residual rows, updated in place);
        returns the last layer's FFN output (the pending residual delta).
        pos0 None = a decode token at the device position."""
        delta = None
        for L in self.layers:
            h = rmsnorm(x, delta, L["attn_norm"], self.eps)
            if L["linear"]:
                p = L["qkvz"](h)
                d = L["out"](self._gdn(L, p, h, decode=pos0 is None))
            else:
                p = L["qkv"](h)
                o = self._attn_decode(L, p) if pos0 is None else self._attn_prefill(L, p, pos0)
                d = L["o"](o)
            if self.reduce_group is not None:
                d = reduce_partials(d, self.reduce_group)
            h2 = rmsnorm(x, d, L["post_norm"], self.eps)
            delta = L["down"](L["gate_up"].swiglu(h2))
            if self.reduce_group is not None:
                delta = reduce_partials(delta, self.reduce_group)
        return delta

    # ---- public ----
    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """Runs a prompt from position 0 (the caches are reset); returns the
        last token's logits (fp32, vocab) and sets the next token to their
        argmax."""
        self.reset()
        cfg, T = self.cfg, ids.numel()
        if T > self.max_len:
            raise ValueError("prompt longer than the cache")
        x = packed_embedding(ids.reshape(-1).to(self.dev), self.embed.data, qtype=self.embed.quantization_type,
                             vocab_size=cfg.vocab_size, dimensions=cfg.hidden_size, dtype=torch.float32)
        x = x.reshape(T, cfg.hidden_size).contiguous()
        delta = self._layers(x, 0)
        last = x[T - 1:].clone()
        hf = rmsnorm(last, delta[T - 1:].contiguous(), self.out_norm, self.eps)
        logits = self.lm_head(hf)[0]
        self.cur_id[:1].copy_(torch.argmax(logits).to(torch.int32).reshape(1))
        self.pos.fill_(T)
        self.n_pos = T
        return logits

    def _decode_body(self) -> torch.Tensor:
        cfg, B = self.cfg, self.batch
        ids = self.cur_id[:B]
        x = packed_embedding(ids, self.embed.data, qtype=self.embed.quantization_type,
                             vocab_size=cfg.vocab_size, dimensions=cfg.hidden_size, dtype=torch.float32)
        x = x.reshape(B, cfg.hidden_size)
        delta = self._layers(x, None)
        hf = rmsnorm(x, delta, self.out_norm, self.eps)
        logits = self.lm_head(hf)
        ids.copy_(torch.argmax(logits, dim=-1).to(torch.int32))
        self.pos.add_(1)
        return logits

    def decode_step(self, token=None) -> torch.Tensor:
        """One decode step, eagerly: feeds ``token`` (an int for every
        sequence, or one int per sequence of the batch; default: the argmax
        of the previous step) at the current position; returns the logits
        (batch x vocab, fp32)."""
        if self.n_pos >= self.max_len:
            raise ValueError("cache full")
        if token is not None:
            if isinstance(token, int):
                self.cur_id[:self.batch].fill_(int(token))
            else:
                t = torch.as_tensor(token, dtype=torch.int32).reshape(-1)
                if t.numel() != self.batch:
                    raise ValueError(f"expected {self.batch} tokens")
                self.cur_id[:self.batch].copy_(t.to(self.dev))
        logits = self._decode_body()
        self.n_pos += 1
        return logits

    def capture_decode(self) -> None:
        """Captures one decode step as a CUDA graph (run one eager step
        first: it sizes the library workspaces, and advances the position)."""
        st = torch.cuda.Stream(device=self.dev)
        st.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        B = self.batch
        saved = [(L["conv_state"][:B].clone(), L["state"][:B].clone()) for L in self.layers if L["linear"]]
        pos, cur = self.pos.clone(), self.cur_id.clone()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                self._graph_logits = self._decode_body()
        torch.cuda.current_stream(self.dev).wait_stream(st)
        # Capture does not execute; restore anyway in case a kernel ran eagerly.
        it = iter(saved)
        for L in self.layers:
            if L["linear"]:
                cs, s = next(it)
                L["conv_state"][:B].copy_(cs)
                L["state"][:B].copy_(s)
        self.pos.copy_(pos)
        self.cur_id.copy_(cur)
        self._graph = g

    def replay_decode(self, n: int = 1) -> None:
        """n decode tokens through the captured graph (greedy)."""
        if self._graph is None:
            raise RuntimeError("capture_decode() first")
        if self.n_pos + n > self.max_len:
            raise ValueError("cache full")
        for _ in range(n):
            self._graph.replay()
        self.n_pos += n

    def release_graph(self) -> None:
        """Drops the captured decode graph (and the memory it holds)."""
        self._graph = None

    @property
    def graph_logits(self) -> torch.Tensor:
        return self._graph_logits


def build_qwen35_head_split(weights: dict, cfg: Qwen35Config | None = None, device="cuda", max_len: int = 2304,
                            group=None, max_batch: int = 1) -> Qwen35:
    """The model split by heads over the ranks of ``group``: this rank's
    weights and configuration from ``head_split_weights``, the blocks'
    partial outputs summed over the ranks (``Qwen35``'s ``reduce_group``).
    Collective: every rank of the group builds its part."""
    cfg = cfg or Qwen35Config()
    world = dist.get_world_size(group) if group is not None else 1
    rank = dist.get_rank(group) if group is not None else 0
    local, local_cfg = head_split_weights(weights, cfg, world, rank)
    return Qwen35(local, local_cfg, device, max_len=max_len, max_batch=max_batch, reduce_group=group)


def build_qwen35(weights: dict, cfg: Qwen35Config | None = None, device="cuda", max_len: int = 2304,
                 group=None, max_batch: int = 1) -> Qwen35:
    """The model from GGUF-named weights (``qwen35.py:104-152``): packed
    projections as ``PackedWeight`` on the device, plain tensors as arrays;
    ``group``: split every packed projection over the group's ranks;
    ``max_batch``: sequences a batched decode can hold (``fork``)."""
    return Qwen35(weights, cfg or Qwen35Config(), device, max_len=max_len, group=group, max_batch=max_batch)
