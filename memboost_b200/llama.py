"""Layer-streaming GPTQ of a Llama-2-shaped decoder -- the caller of the
quantization path (the reference's quantize_llama, models/llama.py:385-659).

Per layer: forward the calibration hidden states through the layer with fp16
weights, accumulating the four input Hessians (llama.py:523-551) on the
tcgen05 kernel; GPTQ + memboost quantize of the seven projections
(llama.py:553-617); then forward the same hidden states through the
quantized layer to produce the next layer's inputs (llama.py:619-632).  With
a communicator the calibration samples are split over the ranks (each
forwards its own) and each layer's GPTQ runs with the tokens and weight rows
split (gptq.quantize_layer_distributed): the layers stay sequential (layer
l + 1's inputs need layer l quantized), the work inside each layer is spread.

No checkpoint or tokenizer exists here: layer weights are seeded N(0, 0.02^2)
draws of the Llama shapes and the calibration hidden states seeded Gaussian
embeddings.  The block's math is the architecture's (RMSNorm, rotary
embeddings in the rotate-half convention, causal attention, SwiGLU).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import gptq
from .ops import dequantize


@dataclass
class LlamaConfig:
    """The reference's LlamaConfig fields (models/llama.py:41-52)."""
    vocab_size: int = 32000
    n_embd: int = 4096
    n_layer: int = 32
    n_head: int = 32
    n_kv_heads: int = 32
    n_inner: int = 11008
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_seq_len: int = 2048
    ratio_4bit: float = 0.1


PROJECTIONS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def projection_shape(cfg: LlamaConfig, name: str) -> tuple[int, int]:
    hd = cfg.n_embd // cfg.n_head
    return {"self_attn.q_proj": (cfg.n_embd, cfg.n_embd),
            "self_attn.k_proj": (cfg.n_kv_heads * hd, cfg.n_embd),
            "self_attn.v_proj": (cfg.n_kv_heads * hd, cfg.n_embd),
            "self_attn.o_proj": (cfg.n_embd, cfg.n_embd),
            "mlp.gate_proj": (cfg.n_inner, cfg.n_embd),
            "mlp.up_proj": (cfg.n_inner, cfg.n_embd),
            "mlp.down_proj": (cfg.n_embd, cfg.n_inner)}[name]


def layer_weights(cfg: LlamaConfig, layer: int, device, seed: int = 7) -> dict:
    """fp32 weights of one synthetic layer (seeded per layer and projection)."""
    out = {}
    for j, name in enumerate(PROJECTIONS):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 100003 + layer * 101 + j)
        out[name] = torch.randn(projection_shape(cfg, name), generator=g, device=device) * 0.02
    return out


def calibration_hidden(cfg: LlamaConfig, n_samples: int, seq_len: int, device,
                       seed: int = 3) -> torch.Tensor:
    """[n_samples, seq_len, n_embd] fp16 stand-ins for the token embeddings."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn((n_samples, seq_len, cfg.n_embd), generator=g, device=device)
            * 0.02).to(torch.float16)


def rms_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm with unit weight, computed in fp32 and returned in x's dtype."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def rope_tables(head_dim: int, seq_len: int, theta: float, device):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    ang = torch.outer(torch.arange(seq_len, device=device).float(), inv)
    return ang.cos(), ang.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    T, half = x.shape[2], x.shape[-1] // 2
    c, s = cos[:T][None, None], sin[:T][None, None]
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).to(x.dtype)


def block_forward(cfg: LlamaConfig, x: torch.Tensor, linear: dict, cos, sin,
                  capture: dict | None = None) -> torch.Tensor:
    """One decoder block.  ``linear``: projection name -> callable(x) -> x W^T.
    ``capture`` receives the four projection inputs whose Hessians GPTQ needs
    ("attn": q/k/v input, "o": o_proj input, "mlp": gate/up input, "down":
    down_proj input)."""
    B, T, _ = x.shape
    hd = cfg.n_embd // cfg.n_head
    a_in = rms_norm(x, cfg.rms_norm_eps)
    q = linear["self_attn.q_proj"](a_in).view(B, T, cfg.n_head, hd).transpose(1, 2)
    k = linear["self_attn.k_proj"](a_in).view(B, T, cfg.n_kv_heads, hd).transpose(1, 2)
    v = linear["self_attn.v_proj"](a_in).view(B, T, cfg.n_kv_heads, hd).transpose(1, 2)
    q, k = _rotate(q, cos, sin), _rotate(k, cos, sin)
    rep = cfg.n_head // cfg.n_kv_heads
    if rep > 1:
        k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
    y = F.scaled_dot_product_attention(q, k, v, is_causal=T > 1, scale=1.0 / math.sqrt(hd))
    o_in = y.transpose(1, 2).reshape(B, T, -1)
    x = x + linear["self_attn.o_proj"](o_in)
    m_in = rms_norm(x, cfg.rms_norm_eps)
    d_in = F.silu(linear["mlp.gate_proj"](m_in)) * linear["mlp.up_proj"](m_in)
    x = x + linear["mlp.down_proj"](d_in)
    if capture is not None:
        for key, val in (("attn", a_in), ("o", o_in), ("mlp", m_in), ("down", d_in)):
            capture[key](val)
    return x


def _fp16_linears(w: dict) -> dict:
    wh = {k: v.to(torch.float16) for k, v in w.items()}
    return {k: (lambda x, W=W: F.linear(x.to(torch.float16), W)) for k, W in wh.items()}


def _quantized_linears(q: dict) -> dict:
    deq = {k: dequantize(qt) for k, qt in q.items()}
    return {k: (lambda x, W=W: F.linear(x.to(torch.float16), W)) for k, W in deq.items()}


def quantize_llama_synthetic(cfg: LlamaConfig, n_samples: int = 128, seq_len: int = 2048,
                             device=None, comm=None, seed: int = 7, batch: int = 4,
                             n_layers: int | None = None):
    """Layer-streaming GPTQ of a synthetic Llama (``n_layers`` of cfg's, all
    by default).  With ``comm`` (rowsplit.DistComm / LocalComm) rank r forwards
    samples r, r + world, ...; every rank ends with every layer's tensors.
    Returns (quantized layers by name, stats with per-layer seconds)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    n_layers = cfg.n_layer if n_layers is None else n_layers
    rank, world = (0, 1) if comm is None else (comm.rank, comm.world)
    hidden = calibration_hidden(cfg, n_samples, seq_len, device)[rank::world].contiguous()
    cos, sin = rope_tables(cfg.n_embd // cfg.n_head, seq_len, cfg.rope_theta, device)
    out, per_layer = {}, []
    fp16_bytes = quant_bytes = 0
    for layer in range(n_layers):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        w = layer_weights(cfg, layer, device, seed)
        accs = {key: gptq.HessianAccumulator(K, device) for key, K in
                (("attn", cfg.n_embd), ("o", cfg.n_embd), ("mlp", cfg.n_embd),
                 ("down", cfg.n_inner))}
        inputs = {}
        lin = _fp16_linears(w)
        with torch.no_grad():
            for s0 in range(0, hidden.shape[0], batch):
                block_forward(cfg, hidden[s0:s0 + batch], lin, cos, sin,
                              capture={k: a.add for k, a in accs.items()})
        if comm is None:
            # the inverses beside the GPTQ updates (largest Hessian first)
            workers = gptq.InverseWorkers(device, workers=len(accs))
            try:
                for key in sorted(accs, key=lambda k: -accs[k].K):
                    workers.start(key, accs[key].finalize())
                q = {}
                for name in sorted(w, key=lambda n: accs[gptq.LAYER_INPUTS[n]].K):
                    h_diag, hc = workers.take(gptq.LAYER_INPUTS[name])
                    q[name] = gptq.make_quantized_linear(w[name], h_diag, hc,
                                                         cfg.ratio_4bit).q_weight
            finally:
                workers.close()
            q = {name: q[name] for name in w}
        else:
            # the accumulated sums over this rank's tokens, reduced inside
            tokens = torch.tensor([float(accs["attn"].tokens)], dtype=torch.float64,
                                  device=device)
            total = float(comm.all_reduce_sum(tokens).item())
            inv = {}
            for i, (key, acc) in enumerate(accs.items()):
                H = comm.all_reduce_sum(acc.H)
                H.div_(total)
                owner = i % world
                if rank == owner:
                    h_diag, hc = gptq.gptq_inverse(H)
                else:
                    h_diag = torch.empty((acc.K,), dtype=torch.float32, device=device)
                    hc = torch.empty((acc.K, acc.K), dtype=torch.float32, device=device)
                inv[key] = (comm.broadcast(h_diag, owner), comm.broadcast(hc, owner))
            q = gptq.quantize_layer_distributed(w, inputs, comm, cfg.ratio_4bit, inverses=inv)
        del accs
        qlin = _quantized_linears(q)
        with torch.no_grad():
            nxt = torch.empty_like(hidden)
            for s0 in range(0, hidden.shape[0], batch):
                nxt[s0:s0 + batch] = block_forward(cfg, hidden[s0:s0 + batch], qlin, cos, sin)
        hidden = nxt
        for name, qt in q.items():
            out[f"layers.{layer}.{name}"] = qt
            fp16_bytes += qt.M * qt.K * 2
            quant_bytes += qt.total_bytes
        torch.cuda.synchronize(device)
        per_layer.append(time.perf_counter() - t0)
    return out, {"seconds_per_layer": per_layer, "fp16_bytes": fp16_bytes,
                 "quantized_bytes": quant_bytes,
                 "compression_ratio": fp16_bytes / max(1, quant_bytes)}
