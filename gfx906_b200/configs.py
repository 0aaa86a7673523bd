"""The benchmark configurations and their seeded synthetic inputs.

C1..C5 are the five workloads the path is measured on (fp16 [B,H,S,D],
no mask, scale 1/sqrt(D)). Inputs are iid N(0,1) (times 0.5 for C3), drawn on
the CPU in fp32 from a seeded ``torch.Generator`` and rounded to fp16, so that
every device and the CPU oracle see identical bits.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class AttnConfig:
    name: str
    B: int
    H: int
    Sq: int
    Skv: int
    D: int
    seed: int
    std: float = 1.0

    @property
    def scale(self) -> float:
        return self.D ** -0.5

    @property
    def flops(self) -> float:
        """4*B*H*Sq*Skv*D (QK^T and PV multiply-adds, 2 flops each)."""
        return 4.0 * self.B * self.H * self.Sq * self.Skv * self.D

    @property
    def io_bytes(self) -> int:
        """Bytes of Q, K, V and O in fp16 (the minimum HBM traffic of one call)."""
        return 2 * self.B * self.H * self.D * (2 * self.Sq + 2 * self.Skv)

    def describe(self) -> str:
        return (f"B{self.B} H{self.H} Sq{self.Sq} Skv{self.Skv} D{self.D} fp16, "
                f"N(0,{self.std:g}^2) seed {self.seed}, scale 1/sqrt({self.D})")


CONFIGS = {
    "C1": AttnConfig("C1", 1, 8, 1024, 1024, 64, seed=0),
    "C2": AttnConfig("C2", 1, 24, 4096, 4096, 128, seed=1),
    "C3": AttnConfig("C3", 2, 16, 4096, 1024, 128, seed=2, std=0.5),
    "C4": AttnConfig("C4", 1, 4, 4096, 4096, 512, seed=3),
    "C5": AttnConfig("C5", 1, 1, 131072, 131072, 64, seed=4),
    "C5s": AttnConfig("C5s", 1, 1, 32768, 32768, 64, seed=4),
}


def make_qkv(B, H, Sq, Skv, D, seed=0, std=1.0, device="cpu"):
    """Seeded fp16 q [B,H,Sq,D], k/v [B,H,Skv,D]; drawn on the CPU in fp32."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(B, H, Sq, D, generator=g) * std).half()
    k = (torch.randn(B, H, Skv, D, generator=g) * std).half()
    v = (torch.randn(B, H, Skv, D, generator=g) * std).half()
    if device != "cpu":
        q, k, v = q.to(device), k.to(device), v.to(device)
    return q, k, v


def config_inputs(cfg: AttnConfig, device="cpu"):
    return make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, cfg.seed, cfg.std, device)
