"""Route ViT attention through low-precision attention (reference: src/vit_nvfp4/ptq/qattention.py:20-71).

Registers an attention implementation (``nvfp4_attn``) in the attention-function registry that
HF transformers' attention modules dispatch through (and in vitfp4's own ViT registry), flags the
modules picked by a predicate, and points every attention module's config at the implementation:
flagged modules run ``quant_sdpa``, the rest exact SDPA.
"""
import torch.nn.functional as F

from .policy import block_index, _in_container

_IMPL = "nvfp4_attn"


def _quant_attention(module, query, key, value, attention_mask=None, dropout=0.0, scaling=None,
                     is_causal=None, **kwargs):
    from ..nvfp4.attention import quant_sdpa
    if getattr(module, "_nvfp4_attn", False):
        out = quant_sdpa(query, key, value, attn_mask=attention_mask, is_causal=bool(is_causal), scale=scaling,
                         qk=getattr(module, "_nvfp4_qk", "fp8"), pv=getattr(module, "_nvfp4_pv", "fp8"))
    else:
        out = F.scaled_dot_product_attention(query, key, value, attn_mask=attention_mask, dropout_p=dropout,
                                             scale=scaling, is_causal=bool(is_causal))
    return out.transpose(1, 2).contiguous(), None


def vit_attn_policy(num_layers: int, skip_first: int = 2, skip_last: int = 2, container: str | None = None):
    """Predicate picking the attention module (class name contains 'Attention' and it has a
    ``scaling`` attribute) of every middle block."""
    first, stop = skip_first, num_layers - skip_last

    def should(name, module) -> bool:
        if "Attention" not in type(module).__name__ or not hasattr(module, "scaling"):
            return False
        if not _in_container(name, container):
            return False
        idx = block_index(name)
        return idx is not None and first <= idx < stop

    return should


def _register() -> None:
    from .. import vit
    vit.ATTENTION_FUNCTIONS[_IMPL] = _quant_attention
    try:
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        if _IMPL not in ALL_ATTENTION_FUNCTIONS.valid_keys():
            ALL_ATTENTION_FUNCTIONS.register(_IMPL, _quant_attention)
    except Exception:  # transformers absent: vitfp4's own ViT still routes through its registry
        pass


def enable_quant_attention(model, should_quantize_attn, qk: str = "fp8", pv: str = "fp8") -> int:
    """Route attention through ``quant_sdpa`` for the modules matched by ``should_quantize_attn``.
    Returns the number of attention modules flagged."""
    _register()
    n, seen = 0, set()
    for name, mod in model.named_modules():
        if "Attention" in type(mod).__name__ and getattr(mod, "config", None) is not None:
            if id(mod.config) not in seen:
                mod.config._attn_implementation = _IMPL
                seen.add(id(mod.config))
        if should_quantize_attn(name, mod):
            mod._nvfp4_attn, mod._nvfp4_qk, mod._nvfp4_pv = True, qk, pv
            n += 1
    return n
