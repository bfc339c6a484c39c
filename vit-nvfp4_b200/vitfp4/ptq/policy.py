"""Which Linear / attention modules to quantize (reference: src/vit_nvfp4/ptq/policy.py:7-40).

Same selection rule as the reference: a module path carries a transformer-block index
(``layer.N`` / ``layers.N`` / ``blocks.N`` / ``h.N``); the first ``skip_first`` and last
``skip_last`` blocks and every module without a block index stay in bf16.
"""
import re

import torch.nn as nn

BLOCK_INDEX_RE = re.compile(r"(?:^|\.)(?:layer|layers|blocks|h)\.(\d+)(?:\.|$)")


def block_index(name: str):
    """Transformer-block index encoded in a dotted module path, or None."""
    hit = BLOCK_INDEX_RE.search(name)
    return None if hit is None else int(hit.group(1))


def _in_container(name: str, container: str | None) -> bool:
    if container is None:
        return True
    prefix = container + "."
    return name.startswith(prefix) or ("." + prefix) in name


def vit_block_policy(num_layers: int, skip_first: int = 2, skip_last: int = 2, container: str | None = None):
    """Predicate ``(name, module) -> bool`` selecting the nn.Linear layers of the middle blocks."""
    first, stop = skip_first, num_layers - skip_last

    def should_quantize(name: str, module: nn.Module) -> bool:
        if not isinstance(module, nn.Linear) or not _in_container(name, container):
            return False
        idx = block_index(name)
        return idx is not None and first <= idx < stop

    return should_quantize
