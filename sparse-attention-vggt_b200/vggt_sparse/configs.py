"""The benchmark configurations of the sparse global-attention layer.

cfg1  4 frames, top-k 25% of key blocks, 64 centres (CPU-runnable case)
cfg2  32 frames, softmax-mass 0.9, heads 0-3 dense, 128 centres (headline)
cfg3  16 frames, top-k 25% (one layer here; the full aggregator end to end is
      bench.py --component aggregator, the reference's model with this drop-in)
cfg4  100 frames, top-k 15%, 256 centres, head-sharded over 2/4/8 GPUs
cfg5  256 frames, mass 0.85, heads 0-3 dense, 512 centres, query-block sharded
"""
from dataclasses import dataclass, field


@dataclass(frozen=True)
class LayerConfig:
    name: str
    frames: int
    centres: int
    mode: str                    # 'topk' (retention) or 'mass' (tau)
    retention: float = 0.25
    tau: float = 0.9
    dense_heads: tuple = field(default_factory=tuple)
    heads: int = 16
    dim: int = 64
    block: int = 64


CONFIGS = {
    "cfg1": LayerConfig("cfg1", frames=4, centres=64, mode="topk", retention=0.25),
    "cfg2": LayerConfig("cfg2", frames=32, centres=128, mode="mass", tau=0.9,
                        dense_heads=(0, 1, 2, 3)),
    "cfg3": LayerConfig("cfg3", frames=16, centres=64, mode="topk", retention=0.25),
    "cfg4": LayerConfig("cfg4", frames=100, centres=256, mode="topk", retention=0.15),
    "cfg5": LayerConfig("cfg5", frames=256, centres=512, mode="mass", tau=0.85,
                        dense_heads=(0, 1, 2, 3)),
}
