"""A seeded PEFT adapter on disk (adapter_config.json + safetensors) with
Mistral-7B module shapes, shared by the pool tests and the script that
records the reference loader's results for it."""

import hashlib
import json
from pathlib import Path

import torch
from safetensors.torch import save_file

HIDDEN, KV_OUT, MLP_INTER = 4096, 1024, 14336
GEOM = {"q_proj": (HIDDEN, HIDDEN), "k_proj": (HIDDEN, KV_OUT), "v_proj": (HIDDEN, KV_OUT),
        "o_proj": (HIDDEN, HIDDEN), "gate_proj": (HIDDEN, MLP_INTER), "up_proj": (HIDDEN, MLP_INTER),
        "down_proj": (MLP_INTER, HIDDEN)}


def tensor_digest(t: torch.Tensor) -> str:
    """sha256 of a 16-bit tensor's bytes."""
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def write_adapter(d: Path, r=16, alpha=32, modules=("q_proj", "v_proj"), layers=(0, 1), rslora=False,
                  seed=0, drop_b=None):
    d.mkdir(parents=True)
    cfg = {"r": r, "lora_alpha": alpha, "target_modules": list(modules), "use_rslora": rslora}
    (d / "adapter_config.json").write_text(json.dumps(cfg))
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for li in layers:
        for m in modules:
            k_in, n_out = GEOM[m]
            parent = "self_attn" if m.endswith(("q_proj", "k_proj", "v_proj", "o_proj")) else "mlp"
            pre = f"base_model.model.model.layers.{li}.{parent}.{m}"
            tensors[f"{pre}.lora_A.weight"] = torch.randn(r, k_in, generator=g) * 0.05
            if drop_b != (li, m):
                tensors[f"{pre}.lora_B.weight"] = torch.randn(n_out, r, generator=g) * 0.05
    # a key that is not a LoRA weight, and a module outside target_modules
    tensors["base_model.model.lm_head.weight"] = torch.zeros(4, 4)
    tensors["base_model.model.model.layers.0.mlp.down_proj.lora_A.weight"] = torch.ones(r, MLP_INTER)
    tensors["base_model.model.model.layers.0.mlp.down_proj.lora_B.weight"] = torch.ones(HIDDEN, r)
    if "down_proj" in modules:
        del tensors["base_model.model.model.layers.0.mlp.down_proj.lora_A.weight"]
        del tensors["base_model.model.model.layers.0.mlp.down_proj.lora_B.weight"]
        g2 = torch.Generator().manual_seed(seed + 1)
        for li in layers:
            pre = f"base_model.model.model.layers.{li}.mlp.down_proj"
            tensors[f"{pre}.lora_A.weight"] = torch.randn(r, MLP_INTER, generator=g2) * 0.05
            tensors[f"{pre}.lora_B.weight"] = torch.randn(HIDDEN, r, generator=g2) * 0.05
    save_file(tensors, str(d / "adapter_model.safetensors"))
    return d, tensors
