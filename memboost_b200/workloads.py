"""Seeded synthetic weights and hessian diagonals with the shapes and value
distributions of the benchmark configurations.

No real checkpoints or calibration data are used: these generators stand in
for Llama-2-7B / Llama-70B-shaped weights.  Everything is drawn on the CPU
from a seeded torch.Generator, so every machine (and the CPU oracle) sees the
same bytes.

  single_4096      4096x4096 fp16 ~ N(0, 0.02^2), seed 0, 0.1% of entries
                   (uniform positions) x10; hessian_diag = ones; ratio 0.1
  mlp_7b           11008x4096 and 4096x11008 ~ N(0, 0.02^2); 0.05% of entries
                   replaced by 0.02 * Student-t(3); hessian_diag per column
                   ~ lognormal(0, 1.5); ratio 0.1
  llama7b_model    32 layers x {q,k,v,o 4096^2, gate/up 11008x4096,
                   down 4096x11008} ~ N(0, 0.02^2); lognormal(0, 1.5) hessian
                   per matrix; ratio 0.1
  mlp_70b          28672x8192 and 8192x28672 ~ N(0, 0.015^2); 0.2% x10
                   outliers; lognormal(0, 2.0) hessian; ratio 0.25
  gptq_layer       one Llama-7B layer's GPTQ: calibration activations of
                   128 x 2048 tokens (bf16, Student-t(4) / sqrt(4096), 1% of
                   channels x20) for the attention (K=4096), o_proj (4096),
                   MLP (4096) and down_proj (11008) inputs; fp32 weights
                   ~ N(0, 0.02^2) of the seven projection shapes; ratio 0.1
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class MatrixCase:
    name: str
    weights: torch.Tensor       # fp16 [M, K] (CPU)
    hessian_diag: torch.Tensor  # fp32 [K] (CPU)
    ratio_4bit: float


def _normal(M: int, K: int, std: float, g: torch.Generator) -> torch.Tensor:
    return (torch.randn(M, K, generator=g, dtype=torch.float32) * std)


def _student_t(n: int, df: int, g: torch.Generator) -> torch.Tensor:
    z = torch.randn(n, generator=g)
    chi2 = (torch.randn(n, df, generator=g) ** 2).sum(1)
    return z / torch.sqrt(chi2 / df)


def _scatter(w: torch.Tensor, frac: float, g: torch.Generator) -> torch.Tensor:
    n = max(1, int(round(w.numel() * frac)))
    return torch.randint(0, w.numel(), (n,), generator=g)


def lognormal(K: int, sigma: float, g: torch.Generator) -> torch.Tensor:
    return torch.exp(torch.randn(K, generator=g) * sigma).float()


def single_4096(seed: int = 0, M: int = 4096, K: int = 4096) -> MatrixCase:
    g = torch.Generator().manual_seed(seed)
    w = _normal(M, K, 0.02, g)
    idx = _scatter(w, 0.001, g)
    w.view(-1)[idx] *= 10.0
    return MatrixCase("single_4096", w.half(), torch.ones(K, dtype=torch.float32), 0.1)


def mlp_matrix(M: int, K: int, seed: int, std: float = 0.02, outlier_frac: float = 0.0005,
               sigma: float = 1.5, ratio: float = 0.1, name: str = "mlp") -> MatrixCase:
    g = torch.Generator().manual_seed(seed)
    w = _normal(M, K, std, g)
    idx = _scatter(w, outlier_frac, g)
    w.view(-1)[idx] = std * _student_t(idx.numel(), 3, g)
    return MatrixCase(name, w.half(), lognormal(K, sigma, g), ratio)


def mlp_7b(seed: int = 1) -> list[MatrixCase]:
    return [mlp_matrix(11008, 4096, seed, name="mlp_7b_up"),
            mlp_matrix(4096, 11008, seed + 1, name="mlp_7b_down")]


def mlp_70b(seed: int = 5) -> list[MatrixCase]:
    out = []
    for i, (M, K) in enumerate(((28672, 8192), (8192, 28672))):
        g = torch.Generator().manual_seed(seed + i)
        w = _normal(M, K, 0.015, g)
        idx = _scatter(w, 0.002, g)
        w.view(-1)[idx] *= 10.0
        out.append(MatrixCase(f"mlp_70b_{i}", w.half(), lognormal(K, 2.0, g), 0.25))
    return out


LLAMA7B_LAYER = (("q_proj", 4096, 4096), ("k_proj", 4096, 4096), ("v_proj", 4096, 4096),
                 ("o_proj", 4096, 4096), ("gate_proj", 11008, 4096), ("up_proj", 11008, 4096),
                 ("down_proj", 4096, 11008))


def llama7b_shapes(n_layers: int = 32) -> list[tuple[str, int, int]]:
    return [(f"layers.{l}.{n}", M, K) for l in range(n_layers) for (n, M, K) in LLAMA7B_LAYER]


def llama7b_matrix(name: str, M: int, K: int, seed: int, device=None) -> MatrixCase:
    """One matrix of the Llama-2-7B-shaped model: N(0, 0.02^2) fp16 weights
    and a lognormal(0, 1.5) hessian_diag, ratio 0.1.  ``device`` (default the
    CPU) is where the values are drawn and kept; a CUDA generator gives other
    (equally distributed) values than the CPU one for the same seed."""
    device = torch.device("cpu") if device is None else torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn((M, K), generator=g, device=device, dtype=torch.float32).mul_(0.02).half()
    h = torch.randn((K,), generator=g, device=device).mul_(1.5).exp_().float()
    return MatrixCase(name, w, h, 0.1)


def llama7b_model_seed(i: int) -> int:
    """Seed of matrix i (in llama7b_shapes order) of the whole-model workload."""
    return 1000 + i


def small_case(M: int, K: int, seed: int, kind: str = "normal") -> MatrixCase:
    """Small seeded inputs for parity tests.

    kinds: normal (N(0, 0.02^2) + lognormal hessian), ones (hessian all ones),
    shifted (some groups entirely positive / negative -> outliers),
    const (constant groups, zero range), ties (repeated column groups so
    sensitivities tie), tiny (hessian spanning 1e-10 .. 1e10).
    """
    g = torch.Generator().manual_seed(seed)
    w = _normal(M, K, 0.02, g)
    h = lognormal(K, 1.5, g)
    ng = (K + 15) // 16
    if kind == "ones":
        h = torch.ones(K)
    elif kind == "shifted":
        shift = torch.zeros(K)
        for gi in range(ng):
            r = int(torch.randint(0, 4, (1,), generator=g))
            shift[gi * 16:(gi + 1) * 16] = (0.0, 0.06, -0.06, 0.2)[r]
        w = w + shift
    elif kind == "const":
        for gi in range(0, ng, 3):
            w[:, gi * 16:(gi + 1) * 16] = float(torch.randn(1, generator=g)) * 0.05
    elif kind == "ties":
        base = w[:, :16].clone()
        for gi in range(ng):
            if (gi * 16 + 16) <= K:
                w[:, gi * 16:gi * 16 + 16] = base
        h = torch.ones(K)
    elif kind == "tiny":
        h = torch.exp(torch.rand(K, generator=g) * 46.0 - 23.0)
        h[torch.rand(K, generator=g) < 0.2] = 1e-10
    elif kind != "normal":
        raise ValueError(kind)
    return MatrixCase(f"{kind}_{M}x{K}", w.half(), h.float(), 0.25)


def calibration_activations(N: int, K: int, seed: int, device=None,
                            dtype: torch.dtype = torch.bfloat16,
                            channel_frac: float = 0.01, channel_scale: float = 20.0
                            ) -> torch.Tensor:
    """[N, K] calibration inputs: Student-t(4) / sqrt(4096), with a seeded
    ``channel_frac`` of the K channels scaled by ``channel_scale`` (the
    outlier channels of LLM activations).  Student-t(4) is drawn as
    Z / sqrt(chi2_4 / 4) from five normals, so it is cheap on any device;
    ``device`` defaults to the CPU (bytes identical for a given seed)."""
    device = torch.device("cpu") if device is None else torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    z = torch.randn((N, K), generator=g, device=device)
    chi2 = torch.zeros((N, K), device=device)
    for _ in range(4):
        chi2.addcmul_(n := torch.randn((N, K), generator=g, device=device), n)
    x = z.div_(chi2.div_(4.0).sqrt_()).div_(64.0)
    gc = torch.Generator()
    gc.manual_seed(seed + 7919)
    n_ch = max(1, int(round(channel_frac * K)))
    ch = torch.randperm(K, generator=gc)[:n_ch].to(device)
    x[:, ch] *= channel_scale
    return x.to(dtype)


GPTQ_LAYER_SHAPES = {  # name -> (M, K) of a Llama-2-7B layer
    "self_attn.q_proj": (4096, 4096), "self_attn.k_proj": (4096, 4096),
    "self_attn.v_proj": (4096, 4096), "self_attn.o_proj": (4096, 4096),
    "mlp.gate_proj": (11008, 4096), "mlp.up_proj": (11008, 4096),
    "mlp.down_proj": (4096, 11008),
}
GPTQ_INPUT_FEATURES = {"attn": 4096, "o": 4096, "mlp": 4096, "down": 11008}


def gptq_layer(seed: int = 11, tokens: int = 128 * 2048, device=None, scale: int = 1):
    """(weights, inputs) of one synthetic Llama-7B layer for GPTQ.  ``scale``
    divides every dimension (shapes stay multiples of 128 for scale <= 8)."""
    device = torch.device("cpu") if device is None else torch.device(device)
    weights = {}
    for i, (name, (M, K)) in enumerate(GPTQ_LAYER_SHAPES.items()):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 100 + i)
        weights[name] = torch.randn((M // scale, K // scale), generator=g, device=device) * 0.02
    inputs = {key: calibration_activations(tokens // scale, K // scale, seed * 1000 + j, device)
              for j, (key, K) in enumerate(GPTQ_INPUT_FEATURES.items())}
    return weights, inputs
