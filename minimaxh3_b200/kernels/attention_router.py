"""Drop-in replacement for the reference's ``kernels/attention_router.py``.

Same public surface and the same routing rules as viragadel6/minimaxh3
``kernels/attention_router.py``: module globals ``enabled`` / ``repair_tau`` /
``min_seq`` (:11-13) set by ``configure`` (:25-28); ``denoiser_scope`` (a
thread-local depth counter, :133-139); ``instrument_transformer`` (:118-130);
``install`` (:105-115), which points ``F.scaled_dot_product_attention`` and
``torch._C._nn.scaled_dot_product_attention`` at ``routed_sdpa``; and
``routed_sdpa`` itself (:56-102), which sends a call to the FP8 kernel only
when every gate holds and otherwise to the SDPA captured at import
(``_orig_sdpa``, :17).  The rules have to match the reference exactly because
the runtime (generator, model manager) relies on them; the FP8 kernel behind
them is this package's.
"""
from __future__ import annotations

import functools
import threading
from contextlib import contextmanager

import torch
import torch.nn.functional as F

from .fp8_attention import fp8_attention, is_supported

enabled: bool = True
repair_tau: float = -1.0
min_seq: int = 4096

_tls = threading.local()
_lock = threading.Lock()
_orig_sdpa = F.scaled_dot_product_attention
_installed: bool = False


def _get_depth() -> int:
    return getattr(_tls, "depth", 0)


def configure(enabled: bool, repair_tau: float, min_seq: int) -> None:
    """Set the three routing knobs (process-global, like the reference)."""
    g = globals()
    g["enabled"] = bool(enabled)
    g["repair_tau"] = float(repair_tau)
    g["min_seq"] = int(min_seq)


def _extract_per_key_mask(attn_mask, B: int, Sk: int, device):
    """Reduce an SDPA mask to one value per (batch, key), if it is one.

    Returns (ok, key_mask, key_bias).  Accepted: no mask; or a tensor on
    ``device`` with 2 to 4 dims whose last two dims are (1, Sk) and whose
    leading dims, left-padded to 4, are (1 or B, 1).  A bool mask becomes
    ``key_mask`` [B,Sk]; a floating mask becomes ``key_bias`` [B,Sk] f32;
    any other dtype or shape is not per-key (ok = False).
    """
    if attn_mask is None:
        return True, None, None
    if not isinstance(attn_mask, torch.Tensor) or attn_mask.device != device:
        return False, None, None
    nd = attn_mask.ndim
    if nd < 2 or nd > 4:
        return False, None, None
    if attn_mask.shape[-2] != 1 or attn_mask.shape[-1] != Sk:
        return False, None, None
    shape4 = (1,) * (4 - nd) + tuple(attn_mask.shape)
    if shape4[0] not in (1, B) or shape4[1] != 1:
        return False, None, None
    per_key = attn_mask.reshape(shape4).expand(B, 1, 1, Sk)[:, 0, 0, :]
    if per_key.dtype == torch.bool:
        return True, per_key.contiguous(), None
    if per_key.is_floating_point():
        return True, None, per_key.to(torch.float32).contiguous()
    return False, None, None


def _fp8_eligible(query, key, value, dropout_p, is_causal, enable_gqa) -> bool:
    return (
        _get_depth() > 0
        and enabled
        and dropout_p == 0.0
        and not is_causal
        and not enable_gqa
        and isinstance(query, torch.Tensor)
        and isinstance(key, torch.Tensor)
        and isinstance(value, torch.Tensor)
        and query.shape[-1] == key.shape[-1] == value.shape[-1]
        and is_supported(query, key, value)
        and query.shape[2] >= min_seq
    )


def routed_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                enable_gqa=False):
    """``F.scaled_dot_product_attention`` with long non-causal calls sent to FP8."""
    if _fp8_eligible(query, key, value, dropout_p, is_causal, enable_gqa):
        ok, key_mask, key_bias = _extract_per_key_mask(attn_mask, query.shape[0], key.shape[2], query.device)
        if ok:
            return fp8_attention(query, key, value, scale=scale, key_mask=key_mask, key_bias=key_bias,
                                 repair_tau=repair_tau)
    return _orig_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal,
                      scale=scale, enable_gqa=enable_gqa)


def install() -> None:
    """Route every SDPA call in the process through ``routed_sdpa`` (idempotent)."""
    global _installed
    with _lock:
        if _installed:
            return
        F.scaled_dot_product_attention = routed_sdpa
        nn_mod = getattr(torch._C, "_nn", None)
        if nn_mod is not None and hasattr(nn_mod, "scaled_dot_product_attention"):
            nn_mod.scaled_dot_product_attention = routed_sdpa
        _installed = True


def instrument_transformer(transformer):
    """Wrap ``transformer.forward`` in ``denoiser_scope`` (once)."""
    if getattr(transformer, "_denoiser_scope_instrumented", False):
        return transformer
    inner = transformer.forward

    @functools.wraps(inner)
    def _scoped_forward(*args, **kwargs):
        with denoiser_scope(transformer):
            return inner(*args, **kwargs)

    transformer.forward = _scoped_forward
    transformer._denoiser_scope_instrumented = True
    return transformer


@contextmanager
def denoiser_scope(transformer=None):
    """Enable FP8 routing on this thread for the duration of the block."""
    _tls.depth = _get_depth() + 1
    try:
        yield transformer
    finally:
        _tls.depth = max(0, _get_depth() - 1)
