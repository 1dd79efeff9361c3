"""The decoder-layer workload: one Llama-style layer forward as the Magnetar Runtime drives
a provider -- one ``submit_kernel`` per graph node, every intermediate resident on the
device (the node sequence of the reference's hot path at batch 1 / seq 128 / hidden 512).

Nodes: embedding -> rmsnorm -> matmul x3 (Q, K, V) -> rope x2 -> causal attention ->
matmul-residual (O projection + residual) -> rmsnorm -> gated-matmul (SwiGLU gate/up) ->
matmul-residual (down projection + residual).  ``capture`` records the whole layer into one
CUDA graph (the reference's step capture) so that a replay is a single launch.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import numpy as np

from .executor import CudaExecutor, KernelInvocation


@dataclass(frozen=True)
class DecoderLayerConfig:
    seq: int = 128
    hidden: int = 512
    heads: int = 8
    head_dim: int = 64
    ffn: int = 1376
    vocab: int = 32000
    rope_theta: float = 10000.0
    eps: float = 1e-5
    weight_std: float = 0.02

    @property
    def flops(self) -> float:
        """Matmul + attention FLOPs of one forward (attention counted causal)."""
        s, h, f = self.seq, self.hidden, self.ffn
        proj = 2 * s * (4 * h * h + 3 * h * f)
        attn = 4 * s * s * self.head_dim * self.heads / 2
        return float(proj + attn)


WEIGHTS = ("table", "attn_norm", "wq", "wk", "wv", "wo", "mlp_norm", "wg", "wu", "wd")


def make_inputs(cfg: DecoderLayerConfig, seed: int = 0) -> Dict[str, np.ndarray]:
    """Seeded synthetic weights N(0, std) and uniform-random token ids (as f32 integers)."""
    rng = np.random.default_rng(seed)
    h, f = cfg.hidden, cfg.ffn

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * cfg.weight_std).astype(np.float32)

    return {
        "table": w(cfg.vocab, h),
        "attn_norm": w(h),
        "wq": w(h, h), "wk": w(h, h), "wv": w(h, h), "wo": w(h, h),
        "mlp_norm": w(h),
        "wg": w(h, f), "wu": w(h, f), "wd": w(f, h),
        "ids": rng.integers(0, cfg.vocab, size=(cfg.seq,)).astype(np.float32),
    }


def invocations(cfg: DecoderLayerConfig, prefix: str = "") -> List[KernelInvocation]:
    """The layer's node sequence; resource ids are ``prefix`` + name."""
    p = prefix
    rope = {"base": float(cfg.rope_theta), "dimension": cfg.head_dim, "head_count": cfg.heads,
            "position_offset": 0}
    return [
        KernelInvocation("embedding", [p + "table", p + "ids"], p + "x"),
        KernelInvocation("rmsnorm", [p + "x", p + "attn_norm"], p + "h", {"epsilon": float(cfg.eps)}),
        KernelInvocation("matmul", [p + "h", p + "wq"], p + "q"),
        KernelInvocation("matmul", [p + "h", p + "wk"], p + "k"),
        KernelInvocation("matmul", [p + "h", p + "wv"], p + "v"),
        KernelInvocation("rope", [p + "q"], p + "qr", rope),
        KernelInvocation("rope", [p + "k"], p + "kr", rope),
        KernelInvocation("attention", [p + "qr", p + "kr", p + "v"], p + "a",
                         {"head_count": cfg.heads, "head_dimension": cfg.head_dim, "causal": True}),
        KernelInvocation("matmul-residual", [p + "a", p + "wo", p + "x"], p + "x2"),
        KernelInvocation("rmsnorm", [p + "x2", p + "mlp_norm"], p + "h2", {"epsilon": float(cfg.eps)}),
        KernelInvocation("gated-matmul", [p + "h2", p + "wg", p + "wu"], p + "g"),
        KernelInvocation("matmul-residual", [p + "g", p + "wd", p + "x2"], p + "out"),
    ]


def load(ex: CudaExecutor, inputs: Dict[str, np.ndarray], prefix: str = "") -> None:
    for name in WEIGHTS:
        ex.write_weight_tensor(prefix + name, inputs[name])
    ex.write_tensor(prefix + "ids", inputs["ids"])


def forward(ex: CudaExecutor, cfg: DecoderLayerConfig, prefix: str = "") -> None:
    for inv in invocations(cfg, prefix):
        ex.run(inv)


def capture(ex: CudaExecutor, cfg: DecoderLayerConfig, prefix: str = "") -> None:
    """Runs the layer once (allocating every intermediate), then records it as one graph."""
    forward(ex, cfg, prefix)
    ex.synchronize()
    ex.begin_step_capture()
    try:
        forward(ex, cfg, prefix)
    except Exception:
        ex.abort_step_capture()
        raise
    ex.end_step_capture()
