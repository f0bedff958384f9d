"""The pieces of the reference ``fused_linear`` module (scripts/fused_linear.py) that the fused MLP
path uses: LoRA-layer decomposition, the per-step bf16 cast cache and the path counters.

``fused_mlp`` imports ``STATS``, ``_cast`` and ``_part`` from here exactly as the reference does
(scripts/fused_mlp.py:27); the training step calls ``new_step()`` at the start of every step.
"""
from torch import nn

_THIN = 64
STATS = {"gộp": 0, "gọi thẳng": 0}


def _part(m):
    """(base Linear, A, B, scaling) of a PEFT LoRA Linear, (m, None, None, 1.0) for a plain frozen Linear,
    None when the layer cannot take the fused path (scripts/fused_linear.py:30-48)."""
    base = getattr(m, "base_layer", None)
    if base is None:
        if type(m) is nn.Linear and m.bias is None and not m.weight.requires_grad:
            return m, None, None, 1.0
        return None
    if base.bias is not None or base.weight.requires_grad or m.merged or m.disable_adapters:
        return None
    ads = [a for a in m.active_adapters if a in m.lora_A]
    if len(ads) != 1:
        return None
    a = ads[0]
    drop = m.lora_dropout[a]
    if (a in getattr(m, "lora_variant", {}) or m.use_dora.get(a, False) or m.lora_B[a].bias is not None
            or not (isinstance(drop, nn.Identity) or getattr(drop, "p", 1) == 0)):
        return None
    return base, m.lora_A[a].weight, m.lora_B[a].weight, m.scaling[a]


def _mx(base):
    return getattr(base, "_mx_w", None) is not None


# bf16 copies of the LoRA parameters, made once per step (scripts/fused_linear.py:55-69).  The
# optimizer updates parameters in place without bumping _version, so the cache is keyed by id and
# cleared by new_step() at the start of each step.
_CAST = {}


def new_step():
    _CAST.clear()


def _cast(key, make):
    t = _CAST.get(key)
    if t is None:
        t = _CAST[key] = make()
    return t
