"""Named corpus mixtures over local token caches (the role of megagpt-speedrun/data.py:48-410, which
builds Nemotron-CC / FineWeb-Edu / SFT mixtures from object storage): a recipe maps component names
to native cache directories under a local root. ``data.remote`` covers the object-store side -- the
reference's TreeCache splits under an S3 prefix, mirrored and converted once.

``Recipe(name, components={component: (relative_cache_dir, weight)})``; ``recipe.data_config(root)``
gives a ``DataConfig(source="mixture")`` over the components that exist (``missing="error"`` raises
instead of dropping absent ones, renormalising nothing -- the block mixture normalises weights).
``tokenize_recipe`` runs the tokenize step for every component from raw text directories.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

from ..config import DataConfig


@dataclass(frozen=True)
class Recipe:
    name: str
    components: dict = field(default_factory=dict)  # name -> (relative dir, weight)

    def data_config(self, root: str, *, seed: int = 0, missing: str = "drop") -> DataConfig:
        comps = []
        for cname, (rel, w) in self.components.items():
            path = os.path.join(root, rel)
            if not os.path.exists(os.path.join(path, "meta.json")):
                if missing == "error":
                    raise FileNotFoundError(f"{self.name}: component {cname} has no token cache at {path}")
                continue
            comps.append((cname, path, float(w)))
        if not comps:
            raise FileNotFoundError(f"{self.name}: no component caches under {root}")
        return DataConfig(source="mixture", components=tuple(comps), seed=seed)


# Quality-tiered web + code + math pretraining mixture (component weights are sampling shares).
PRETRAIN = Recipe("pretrain-web-code-math", {
    "web_high": ("web/high", 0.35), "web_medium_high": ("web/medium_high", 0.2), "web_medium": ("web/medium", 0.15),
    "web_synthetic": ("web/synthetic", 0.1), "code": ("code", 0.12), "math": ("math", 0.08)})
EDU = Recipe("edu", {"edu": ("fineweb_edu", 1.0)})
SFT = Recipe("sft-chat", {"chat": ("sft/chat", 0.7), "reasoning": ("sft/reasoning", 0.3)})
RECIPES = {r.name: r for r in (PRETRAIN, EDU, SFT)}


def tokenize_recipe(recipe: Recipe, raw_root: str, cache_root: str, tokenizer: str = "bytes",
                    sample_count: int | None = None) -> dict:
    from .tokenize import TokenizeConfig, tokenize

    out = {}
    for cname, (rel, _) in recipe.components.items():
        src = os.path.join(raw_root, rel)
        if not os.path.exists(src):
            continue
        out[cname] = tokenize(TokenizeConfig(train_paths=(src,), cache_path=os.path.join(cache_root, rel),
                                             tokenizer=tokenizer, sample_count=sample_count))
    return out
