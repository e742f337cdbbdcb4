"""Record the reference adapter loader's results as sha256 digests.

Runs ONLY where the reference checkout is present (the build container): it
loads the reference's ``persona/adapter_pool.py`` by file path, feeds it the
seeded adapter of ``tests/peft_fixture.py`` (rank 12, alpha 32, so the
folded scale 8/3 is not a power of two) in fp16 and bf16, and a seeded
``load_random_adapter`` call, and writes the digests of every resulting
tensor to ``golden_pool.json`` beside this script.

    python tests/golden/make_golden_pool.py [--ref /path/to/reference]
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from peft_fixture import tensor_digest, write_adapter  # noqa: E402

ADAPTER = dict(r=12, alpha=32, modules=("q_proj", "v_proj", "gate_proj", "down_proj"), layers=(0, 3), seed=11)
RANDOM = dict(slots=3, r=8, seed=3, layers=(0, 31))


def load_ref_pool(ref_root: Path):
    spec = importlib.util.spec_from_file_location("reference_persona_adapter_pool",
                                                  ref_root / "persona" / "adapter_pool.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve their module by name
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PERSONA_REFERENCE_DIR"),
                    required="PERSONA_REFERENCE_DIR" not in os.environ,
                    help="checkout of the reference repository (default: $PERSONA_REFERENCE_DIR)")
    args = ap.parse_args()
    ref = load_ref_pool(Path(args.ref))
    out = {"adapter": {k: list(v) if isinstance(v, tuple) else v for k, v in ADAPTER.items()},
           "random": {k: list(v) if isinstance(v, tuple) else v for k, v in RANDOM.items()}}
    with tempfile.TemporaryDirectory() as td:
        d, _ = write_adapter(Path(td) / "a", **ADAPTER)
        for name, dt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
            cfg, per_layer = ref.load_peft_adapter_tensors(d, dtype=dt)
            out[f"scale_{name}"] = cfg.scale
            out[f"load_{name}"] = {f"{li}.{m}.{ab}": tensor_digest(t)
                                   for li, mods in per_layer.items() for m, pair in mods.items()
                                   for ab, t in zip("AB", pair)}
    pool = ref.AdapterPool(RANDOM["slots"], RANDOM["r"], torch.device("cpu"), torch.float16)
    slot = pool.load_random_adapter("x", generator=torch.Generator().manual_seed(RANDOM["seed"]))
    out["random_slot"] = slot
    out["random"]["digests"] = {f"{li}.{f}": tensor_digest(getattr(pool.layers[li], f)[slot])
                                for li in RANDOM["layers"] for f in ref.LayerPools.__dataclass_fields__}
    (HERE / "golden_pool.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(f"wrote {HERE / 'golden_pool.json'}")


if __name__ == "__main__":
    main()
