"""Shapes and seeds of the decoder-layer and whole-checkpoint fixtures.

Shared by the fixture generator (layer_golden.py) and the GPU parity tests,
so both regenerate the same synthetic weights bit for bit.
"""

from __future__ import annotations

# [out, in] of the seven linears of one Qwen3.5 decoder layer at hidden 5120:
# gated q_proj (40 heads x 128 x 2), 8 KV heads x 128, SwiGLU 17408.
LAYER_LINEARS: dict[str, tuple[int, int]] = {
    "self_attn.q_proj": (10240, 5120),
    "self_attn.k_proj": (1024, 5120),
    "self_attn.v_proj": (1024, 5120),
    "self_attn.o_proj": (5120, 5120),
    "mlp.gate_proj": (17408, 5120),
    "mlp.up_proj": (17408, 5120),
    "mlp.down_proj": (5120, 17408),
}

# Linears that read the same activation share one set of statistics.
LAYER_INPUT_GROUP: dict[str, str] = {
    "self_attn.q_proj": "qkv",
    "self_attn.k_proj": "qkv",
    "self_attn.v_proj": "qkv",
    "self_attn.o_proj": "o",
    "mlp.gate_proj": "gate_up",
    "mlp.up_proj": "gate_up",
    "mlp.down_proj": "down",
}

# One routed expert of the MoE stack: gate/up [768, 2048], down [2048, 768].
EXPERT_LINEARS: dict[str, tuple[int, int]] = {
    "gate_proj": (768, 2048),
    "up_proj": (768, 2048),
    "down_proj": (2048, 768),
}
EXPERT_COUNT = 128

_ORDER = list(LAYER_LINEARS)
_EXPERT_ORDER = list(EXPERT_LINEARS)


def layer_seed(short: str) -> int:
    return 400 + _ORDER.index(short)


def ckpt_layer_seed(short: str) -> int:
    return 500 + _ORDER.index(short)


def expert_seed(expert: int, short: str) -> int:
    return 1000 + 3 * expert + _EXPERT_ORDER.index(short)
