"""patch_model: install the CUDA GDN operators on HF Qwen3.5 modules.

Mirrors the reference's ``patch_model(model, fast_gdn, gdn_v2)`` (src/cb_engine.py:54-77): the
same attributes of ``Qwen3_5GatedDeltaNet`` and the forwards of ``Qwen3_5RMSNormGated`` and of
the layer norm ``Qwen3_5RMSNorm`` are rebound, so HF's own forward (and any engine that calls
those attributes) runs the B200 kernels.
"""
from __future__ import annotations

import types

from . import ops


def patch_model(model, fast_gdn: bool = True, gdn_v2: bool = True):
    """Rebind the GDN plug-in points of every layer of ``model``.

    ``fast_gdn`` / ``gdn_v2`` keep the reference's flag names: with either set, chunked prefill
    goes to the tensor-core kernel (both reference variants compute the same chunk algebra);
    with neither, HF's own chunk fallback stays in place.  The decode recurrence, the decode
    conv update and the gated RMSNorm are always replaced, as the reference always replaces the
    first and the last (src/cb_engine.py:69-77).
    """
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M

    n_gdn = 0
    for m in model.modules():
        if isinstance(m, M.Qwen3_5RMSNorm):
            m.forward = types.MethodType(ops.rmsnorm_forward, m)
        elif isinstance(m, M.Qwen3_5RMSNormGated):
            m.forward = types.MethodType(ops.rmsnorm_gated_forward, m)
        elif isinstance(m, M.Qwen3_5GatedDeltaNet):
            m.recurrent_gated_delta_rule = ops.recurrent_gated_delta_rule
            m.causal_conv1d_update = ops.causal_conv1d_update
            if fast_gdn or gdn_v2:
                m.chunk_gated_delta_rule = ops.chunk_gated_delta_rule
            n_gdn += 1
    return n_gdn
