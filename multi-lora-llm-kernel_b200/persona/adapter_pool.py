"""Adapter pool: PEFT adapter parsing, scale folding and the per-layer slot
pools the BGMV kernels read (drop-in for the reference's
``persona/adapter_pool.py``).

Layout (reference ``persona/adapter_pool.py:112-147``), per decoder layer and
slot dimension S:

* ``A_qkv [S, 3r, 4096]`` -- q, k, v rank blocks stacked along the rank axis
* ``B_q [S, 4096, r]``, ``B_k / B_v [S, 1024, r]``
* ``A_o [S, r, 4096]``, ``B_o [S, 4096, r]``
* ``A_gu [S, 2r, 4096]`` -- gate, up rank blocks; ``B_gate / B_up [S, 14336, r]``
* ``A_down [S, r, 14336]``, ``B_down [S, 4096, r]``

The kernels read A row by row along K and B row by row along R, which is
already the TMA-friendly order, and they take slot / row strides, so the
packed ``A_qkv`` / ``A_gu`` blocks are used in place (see
``persona.model_patch.resolve_a_pool``) instead of being copied out.

On B200 each layer's eleven pools are views into ONE device allocation (a
slab per layer), and loading an adapter stages the whole layer in pinned
host memory and moves it with one host-to-device copy per pool slice.

The LoRA scale ``alpha / r`` (``alpha / sqrt(r)`` with rsLoRA) is folded into
B at load time (reference ``persona/adapter_pool.py:30-34, 98``); no op takes
a scale.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

import torch

# Mistral-7B module geometry (reference persona/adapter_pool.py:13-16)
HIDDEN = 4096
KV_OUT = 1024
MLP_INTER = 14336
NUM_LAYERS = 32

ATTN_SUFFIXES = ("q_proj", "k_proj", "v_proj", "o_proj")
MLP_SUFFIXES = ("gate_proj", "up_proj", "down_proj")

# module -> (A pool, rank block within it, B pool)
MODULE_POOLS = {
    "q_proj": ("A_qkv", 0, "B_q"),
    "k_proj": ("A_qkv", 1, "B_k"),
    "v_proj": ("A_qkv", 2, "B_v"),
    "o_proj": ("A_o", 0, "B_o"),
    "gate_proj": ("A_gu", 0, "B_gate"),
    "up_proj": ("A_gu", 1, "B_up"),
    "down_proj": ("A_down", 0, "B_down"),
}


@dataclass
class AdapterConfig:
    """The fields of a PEFT ``adapter_config.json`` the pool needs."""

    r: int
    lora_alpha: float
    target_modules: List[str]
    use_rslora: bool = False

    @property
    def scale(self) -> float:
        return self.lora_alpha / (self.r ** 0.5 if self.use_rslora else self.r)


def _read_adapter_config(path: Path) -> AdapterConfig:
    raw = json.loads((Path(path) / "adapter_config.json").read_text())
    return AdapterConfig(r=int(raw["r"]), lora_alpha=float(raw["lora_alpha"]),
                         target_modules=list(raw["target_modules"]),
                         use_rslora=bool(raw.get("use_rslora", False)))


def _parse_key(key: str) -> Optional[Tuple[int, str, str]]:
    """``...layers.{i}.{self_attn|mlp}.{module}.lora_{A|B}.weight`` ->
    (layer, module, "A" | "B"); None for any other key."""
    if not key.endswith(".weight"):
        return None
    parts = key.split(".")
    try:
        li = parts.index("layers")
        layer = int(parts[li + 1])
    except (ValueError, IndexError):
        return None
    ab = next((p[-1] for p in parts if p in ("lora_A", "lora_B")), None)
    if ab is None:
        return None
    if "self_attn" in parts:
        module = parts[parts.index("self_attn") + 1]
    elif "mlp" in parts:
        module = parts[parts.index("mlp") + 1]
    else:
        raise ValueError(f"Unrecognized adapter key: {key}")
    return layer, module, ab


def load_peft_adapter_tensors(
    adapter_dir: Path, dtype: torch.dtype = torch.float16,
) -> Tuple[AdapterConfig, Dict[int, Dict[str, Tuple[torch.Tensor, torch.Tensor]]]]:
    """Load one PEFT adapter into ``{layer: {module: (A [r, in], B_scaled [out, r])}}``.

    B is cast to ``dtype`` first and then multiplied by the scale with one
    rounding, the order the reference uses (``persona/adapter_pool.py:72-98``),
    so the pooled bytes are the reference's.  Modules outside
    ``target_modules`` are ignored; an A without its B (or the reverse)
    raises ``ValueError``.
    """
    from safetensors import safe_open

    adapter_dir = Path(adapter_dir)
    cfg = _read_adapter_config(adapter_dir)
    path = adapter_dir / "adapter_model.safetensors"
    if not path.exists():
        raise FileNotFoundError(f"Expected adapter_model.safetensors in {adapter_dir}")
    found: Dict[int, Dict[str, Dict[str, torch.Tensor]]] = {}
    with safe_open(str(path), framework="pt", device="cpu") as f:
        for key in f.keys():
            parsed = _parse_key(key)
            if parsed is None:
                continue
            layer, module, ab = parsed
            if module not in cfg.target_modules:
                continue
            t = f.get_tensor(key).to(dtype)
            if ab == "B":
                t = (t.float() * cfg.scale).to(dtype)
            found.setdefault(layer, {}).setdefault(module, {})[ab] = t
    out: Dict[int, Dict[str, Tuple[torch.Tensor, torch.Tensor]]] = {}
    for layer, mods in found.items():
        for module, d in mods.items():
            if "A" not in d or "B" not in d:
                raise ValueError(f"Missing A or B for layer {layer} {module}")
            out.setdefault(layer, {})[module] = (d["A"], d["B"])
    return cfg, out


@dataclass
class LayerPools:
    """Per-decoder-layer pool tensors (one slot dimension S)."""

    A_qkv: torch.Tensor
    B_q: torch.Tensor
    B_k: torch.Tensor
    B_v: torch.Tensor
    A_o: torch.Tensor
    B_o: torch.Tensor
    A_gu: torch.Tensor
    B_gate: torch.Tensor
    B_up: torch.Tensor
    A_down: torch.Tensor
    B_down: torch.Tensor


def pool_shapes(slots: int, r: int, geometry: Tuple[int, int, int] = (HIDDEN, KV_OUT, MLP_INTER)
                ) -> Dict[str, Tuple[int, int, int]]:
    """Pool shapes for ``geometry`` = (hidden, k/v output, MLP intermediate);
    Mistral-7B by default.  q and o keep the hidden width."""
    h, kv, inter = geometry
    return {
        "A_qkv": (slots, 3 * r, h), "B_q": (slots, h, r), "B_k": (slots, kv, r),
        "B_v": (slots, kv, r), "A_o": (slots, r, h), "B_o": (slots, h, r),
        "A_gu": (slots, 2 * r, h), "B_gate": (slots, inter, r), "B_up": (slots, inter, r),
        "A_down": (slots, r, inter), "B_down": (slots, h, r),
    }


def _align(n: int, a: int = 128) -> int:
    return (n + a - 1) // a * a


def _empty_layer_pools(slots: int, r: int, device: torch.device, dtype: torch.dtype,
                       geometry: Tuple[int, int, int] = (HIDDEN, KV_OUT, MLP_INTER)) -> LayerPools:
    """Zeroed pools of one layer, carved out of a single allocation; every
    pool starts on a 256-byte boundary (TMA wants 16)."""
    shapes = pool_shapes(slots, r, geometry)
    sizes = {k: s[0] * s[1] * s[2] for k, s in shapes.items()}
    total = sum(_align(n) for n in sizes.values())
    slab = torch.zeros(total, dtype=dtype, device=device)
    views, off = {}, 0
    for f in fields(LayerPools):
        n = sizes[f.name]
        views[f.name] = slab[off:off + n].view(shapes[f.name])
        off += _align(n)
    return LayerPools(**views)


class AdapterPool:
    """All adapters resident in HBM; a slot table without paging (reference
    ``persona/adapter_pool.py:150-282``).  ``num_layers`` defaults to the
    Mistral-7B 32 and exists so small models and tests can use fewer;
    ``geometry`` (hidden, k/v output, MLP intermediate) likewise defaults to
    Mistral-7B."""

    def __init__(self, max_slots: int, r: int, device: torch.device, dtype: torch.dtype = torch.float16,
                 num_layers: int = NUM_LAYERS, geometry: Tuple[int, int, int] = (HIDDEN, KV_OUT, MLP_INTER)):
        self.max_slots = max_slots
        self.r = r
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_layers = num_layers
        self.geometry = tuple(geometry)
        self.layers: List[LayerPools] = [_empty_layer_pools(max_slots, r, self.device, dtype, self.geometry)
                                         for _ in range(num_layers)]
        self.slot_to_name: Dict[int, str] = {}
        self.name_to_slot: Dict[str, int] = {}
        # popped from the end: slots are handed out max_slots-1, max_slots-2, ...
        self._free_slots: List[int] = list(range(max_slots))

    # ---- slot table ------------------------------------------------------
    def acquire_slot(self, name: str) -> int:
        if name in self.name_to_slot:
            return self.name_to_slot[name]
        if not self._free_slots:
            raise RuntimeError("AdapterPool: no free slots")
        slot = self._free_slots.pop()
        self.name_to_slot[name] = slot
        self.slot_to_name[slot] = name
        return slot

    def release_slot(self, name: str) -> None:
        slot = self.name_to_slot.pop(name, None)
        if slot is None:
            return
        del self.slot_to_name[slot]
        self._free_slots.append(slot)

    # ---- loading -----------------------------------------------------------
    def load_adapter(self, name: str, adapter_dir: Path) -> int:
        """Pack a PEFT adapter into a slot of every layer; returns the slot."""
        cfg, per_layer = load_peft_adapter_tensors(adapter_dir, dtype=self.dtype)
        if cfg.r != self.r:
            raise ValueError(f"Adapter rank {cfg.r} != pool rank {self.r}")
        slot = self.acquire_slot(name)
        for layer_idx in range(self.num_layers):
            self.pack_layer(layer_idx, slot, per_layer.get(layer_idx, {}))
        return slot

    def pack_layer(self, layer_idx: int, slot: int,
                   mods: Dict[str, Tuple[torch.Tensor, torch.Tensor]]) -> None:
        """Write one layer's ``{module: (A [r, in], B [out, r])}`` into ``slot``.
        Modules not given keep what the slot held (zeros for a fresh pool)."""
        pools = self.layers[layer_idx]
        r = self.r
        pin = self.device.type == "cuda"
        for module, (a, b) in mods.items():
            a_name, block, b_name = MODULE_POOLS[module]
            a_dst = getattr(pools, a_name)[slot, block * r:(block + 1) * r]
            b_dst = getattr(pools, b_name)[slot]
            if tuple(a.shape) != tuple(a_dst.shape) or tuple(b.shape) != tuple(b_dst.shape):
                raise ValueError(f"{module}: A {tuple(a.shape)} / B {tuple(b.shape)} do not fit "
                                 f"{tuple(a_dst.shape)} / {tuple(b_dst.shape)}")
            for src, dst in ((a, a_dst), (b, b_dst)):
                src = src.to(self.dtype).contiguous()
                if pin and src.device.type == "cpu":
                    src = src.pin_memory()
                dst.copy_(src, non_blocking=pin)
        if pin:
            torch.cuda.current_stream(self.device).synchronize()

    def load_random_adapter(self, name: str, generator: Optional[torch.Generator] = None) -> int:
        """Random weights of real-adapter shapes (N(0, 1) x 0.01) in a slot.

        Draws happen per layer, per pool, in the pool field order, each the
        size of one slot, as in the reference (``persona/adapter_pool.py:
        243-269``), so the same generator yields the same weights."""
        slot = self.acquire_slot(name)
        for pools in self.layers:
            for f in fields(LayerPools):
                dest = getattr(pools, f.name)[slot]
                dest.copy_(torch.randn(dest.shape, device=self.device, dtype=self.dtype,
                                       generator=generator) * 0.01)
        return slot

    def clear_slot(self, slot: int) -> None:
        """Zero ``slot`` in every pool of every layer (a slot handed to a new
        adapter must not keep modules of the one before)."""
        for pools in self.layers:
            for f in fields(LayerPools):
                getattr(pools, f.name)[slot].zero_()

    def a_pool(self, layer_idx: int, module: str) -> torch.Tensor:
        """``[S, r, K]`` A view of one module (a rank block of a packed pool)."""
        a_name, block, _ = MODULE_POOLS[module]
        return getattr(self.layers[layer_idx], a_name)[:, block * self.r:(block + 1) * self.r]

    def b_pool(self, layer_idx: int, module: str) -> torch.Tensor:
        return getattr(self.layers[layer_idx], MODULE_POOLS[module][2])

    def nbytes(self) -> int:
        return sum(getattr(lp, f.name).numel() * getattr(lp, f.name).element_size()
                   for lp in self.layers for f in fields(LayerPools))


class AdapterCache:
    """More adapters than the pool has slots: LRU paging of the GPU slots.

    The reference's pool keeps every adapter resident ("Version 1 ... without
    LRU paging", reference ``persona/adapter_pool.py:151``).  Here adapters
    are registered by name (a PEFT directory, read once, or in-memory
    ``{layer: {module: (A [r, in], B [out, r])}}`` tensors, scale already
    folded); each keeps a pinned host copy, and ``acquire`` makes the
    adapters of one batch resident: a miss takes a free slot or evicts the
    least recently used adapter that the batch does not use, zeroes that slot
    and copies the adapter in on the current stream (behind any work already
    queued that still reads the old contents).
    """

    def __init__(self, pool: AdapterPool):
        self.pool = pool
        self._host: Dict[str, Dict[int, Dict[str, Tuple[torch.Tensor, torch.Tensor]]]] = {}
        self._lru: List[str] = []  # resident adapters, least recently used first
        self.hits = 0
        self.misses = 0
        self.evictions = 0

    def register(self, name: str, adapter_dir: Optional[Path] = None,
                 layers: Optional[Dict[int, Dict[str, Tuple[torch.Tensor, torch.Tensor]]]] = None) -> None:
        if (adapter_dir is None) == (layers is None):
            raise ValueError("register: give exactly one of adapter_dir and layers")
        if adapter_dir is not None:
            cfg, layers = load_peft_adapter_tensors(Path(adapter_dir), dtype=self.pool.dtype)
            if cfg.r != self.pool.r:
                raise ValueError(f"Adapter rank {cfg.r} != pool rank {self.pool.r}")
        pin = self.pool.device.type == "cuda"
        host = {}
        for li, mods in layers.items():
            if not 0 <= li < self.pool.num_layers:
                raise ValueError(f"{name}: layer {li} outside the pool")
            host[li] = {m: tuple((t.to(self.pool.dtype).contiguous().cpu().pin_memory() if pin
                                  else t.to(self.pool.dtype).contiguous().cpu()) for t in ab)
                        for m, ab in mods.items()}
        self._host[name] = host
        if name in self.pool.name_to_slot:  # re-registered while resident: refresh the slot
            self._load(name, self.pool.name_to_slot[name])

    @property
    def registered(self) -> List[str]:
        return list(self._host)

    @property
    def resident(self) -> List[str]:
        """Resident adapters, least recently used first."""
        return list(self._lru)

    def acquire(self, names: Sequence[str]) -> List[int]:
        """Slots of ``names`` (one batch; repeats allowed), loading misses."""
        want = list(dict.fromkeys(names))
        for n in want:
            if n not in self._host:
                raise KeyError(f"adapter {n!r} is not registered")
        if len(want) > self.pool.max_slots:
            raise RuntimeError(f"a batch of {len(want)} adapters does not fit {self.pool.max_slots} slots")
        for n in want:
            if n in self.pool.name_to_slot:
                self.hits += 1
                self._lru.remove(n)
            else:
                self.misses += 1
                if not self.pool._free_slots:
                    victims = [v for v in self._lru if v not in want]
                    if not victims:
                        raise RuntimeError("no slot can be freed: every slot holds an adapter of this batch or "
                                           "one loaded into the pool directly")
                    victim = victims[0]
                    self._lru.remove(victim)
                    self.pool.release_slot(victim)
                    self.evictions += 1
                slot = self.pool.acquire_slot(n)
                self.pool.clear_slot(slot)
                self._load(n, slot)
            self._lru.append(n)
        return [self.pool.name_to_slot[n] for n in names]

    def _load(self, name: str, slot: int) -> None:
        for li, mods in self._host[name].items():
            self.pool.pack_layer(li, slot, mods)


def validate_uniform_adapters(adapter_dirs: Sequence[Path]) -> AdapterConfig:
    """All adapters must share r, lora_alpha and target_modules (the pool has
    one rank and one folded scale per adapter, reference
    ``persona/adapter_pool.py:272-282``)."""
    configs = [_read_adapter_config(Path(p)) for p in adapter_dirs]
    first = configs[0]
    for c in configs[1:]:
        if c.r != first.r or c.lora_alpha != first.lora_alpha:
            raise ValueError("Adapters must share r and lora_alpha")
        if sorted(c.target_modules) != sorted(first.target_modules):
            raise ValueError("Adapters must share target_modules")
    return first
