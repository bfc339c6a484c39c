"""Accuracy metrics (reference: src/vit_nvfp4/ptq/diagnostics.py:5-42)."""
import torch
import torch.nn.functional as F


@torch.no_grad()
def tensor_cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    """Cosine similarity of two tensors taken as flat fp32 vectors."""
    return float(F.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0))


@torch.no_grad()
def block_output_cosines(ref_model, quant_model, inputs, block_container=None) -> list[float]:
    """Cosine between the outputs of block i of ``ref_model`` and of ``quant_model``, for every block.

    ``inputs``: keyword arguments given to both models (a tensor is passed positionally).  The blocks
    are the children of the module named ``block_container`` in each model (found with
    ``find_block_container`` when None); both models run once with forward hooks on their blocks.
    A block that returns a tuple is measured on its first element.  Locates where a converted model
    departs from its reference."""
    if block_container is None:
        from .models import find_block_container
        block_container = find_block_container(ref_model)
    pairs = list(zip(ref_model.get_submodule(block_container), quant_model.get_submodule(block_container)))
    outs = ({}, {})

    def keep(store, i):
        def hook(_m, _args, out):
            store[i] = (out[0] if isinstance(out, tuple) else out).detach()
        return hook

    hooks = [blk.register_forward_hook(keep(outs[side], i))
             for i, pair in enumerate(pairs) for side, blk in enumerate(pair)]
    try:
        for m in (ref_model, quant_model):
            m(**inputs) if isinstance(inputs, dict) else m(inputs)
    finally:
        for h in hooks:
            h.remove()
    return [tensor_cosine(outs[0][i], outs[1][i]) for i in range(len(pairs))]
