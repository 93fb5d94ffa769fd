"""CPU checks of the slot engine's host-side argument validation (CBEngine.prefill_batch and
decode_step raise before any device work, so a stand-in ``self`` without pools is enough)."""
import types

import pytest
import torch

from conftest import pkg


def _fake():
    return types.SimpleNamespace(N=4, T=64, lens=[0] * 4)


def test_prefill_batch_rejects_a_slot_given_twice():
    eng = pkg("engine")
    ids = [torch.zeros(1, 3, dtype=torch.long)] * 2
    with pytest.raises(ValueError, match="more than once"):
        eng.CBEngine.prefill_batch(_fake(), [1, 1], ids)


def test_decode_step_rejects_a_slot_given_twice_and_a_token_count_mismatch():
    eng = pkg("engine")
    with pytest.raises(ValueError, match="more than once"):
        eng.CBEngine.decode_step(_fake(), [2, 0, 2], [5, 6, 7])
    with pytest.raises(ValueError, match="tokens for"):
        eng.CBEngine.decode_step(_fake(), [0, 1], [5])
