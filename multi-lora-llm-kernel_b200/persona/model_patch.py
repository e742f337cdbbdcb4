"""Replace the targeted linears of a Mistral-style model with MultiLoRALinear
(drop-in for the reference's ``persona/model_patch.py``).

Difference from the reference: ``resolve_a_pool`` returns a VIEW of the
packed ``A_qkv`` / ``A_gu`` pools (the kernels take slot and row strides),
where the reference copies each rank block out at patch time
(``persona/model_patch.py:35-58``).  Adapters loaded into the pool after
patching are therefore seen by the patched layers, and the A pools take no
second copy of HBM.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from persona.adapter_pool import MODULE_POOLS, AdapterPool, LayerPools
from persona.lora_layer import LoRAContext, MultiLoRALinear, make_slot_hook

_PARENT = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn", "o_proj": "self_attn",
           "gate_proj": "mlp", "up_proj": "mlp", "down_proj": "mlp"}


def _attn_mlp_paths() -> List[Tuple[str, str, str]]:
    """(module path within a decoder layer, A pool, B pool), in the
    reference's order (``persona/model_patch.py:14-28``)."""
    return [(f"{_PARENT[m]}.{m}", a, b) for m, (a, _, b) in MODULE_POOLS.items()]


def _module_name_from_path(mod_path: str) -> str:
    return mod_path.rsplit(".", 1)[-1]


def resolve_a_pool(layer_pools: LayerPools, a_key: str, b_key: str, r: int) -> torch.Tensor:
    """``[S, r, K]`` A pool of one module: a rank block of ``A_qkv`` / ``A_gu``
    selected by its B pool, or ``A_o`` / ``A_down`` as they are.  A view,
    never a copy."""
    raw = getattr(layer_pools, a_key)
    blocks = {("A_qkv", "B_q"): 0, ("A_qkv", "B_k"): 1, ("A_qkv", "B_v"): 2,
              ("A_gu", "B_gate"): 0, ("A_gu", "B_up"): 1}
    if a_key in ("A_qkv", "A_gu"):
        if (a_key, b_key) not in blocks:
            raise ValueError(f"Unexpected b_key for {a_key}: {b_key}")
        i = blocks[(a_key, b_key)]
        return raw[:, i * r:(i + 1) * r, :]
    return raw


# The reference's private name, kept for callers that import it.
_resolve_a_pool = resolve_a_pool


def patch_model_with_pools(model: nn.Module, pool: AdapterPool, ctx: LoRAContext,
                           target_modules: Optional[Sequence[str]] = None) -> nn.Module:
    """Wrap the targeted linears of every ``model.model.layers[i]`` with
    ``MultiLoRALinear`` over layer i's pools, and register the slot pre-hook
    once.  Re-entrant: already wrapped linears are left alone."""
    allow = set(target_modules) if target_modules is not None else None
    for layer_idx, block in enumerate(model.model.layers):
        lp = pool.layers[layer_idx]
        for mod_path, a_key, b_key in _attn_mlp_paths():
            if allow is not None and _module_name_from_path(mod_path) not in allow:
                continue
            parent, attr = _rsplit_once(block, mod_path)
            base = getattr(parent, attr, None)
            if not isinstance(base, nn.Module) or isinstance(base, MultiLoRALinear):
                continue
            setattr(parent, attr, MultiLoRALinear(base, ctx, resolve_a_pool(lp, a_key, b_key, pool.r),
                                                  getattr(lp, b_key)))
    if not getattr(model, "_persona_slot_hook", False):
        model.register_forward_pre_hook(make_slot_hook(ctx), with_kwargs=True)
        model._persona_slot_hook = True
    return model


def _rsplit_once(root: nn.Module, path: str) -> Tuple[nn.Module, str]:
    parts = path.split(".")
    cur = root
    for p in parts[:-1]:
        cur = getattr(cur, p)
    return cur, parts[-1]


def _set_module(root: nn.Module, path: str, module: nn.Module) -> None:
    parent, attr = _rsplit_once(root, path)
    setattr(parent, attr, module)
