"""Host checks of the Hugging Face packed cache's supported call pattern
(kvquant.hf_cache): decode steps with a padded mask, another attention scaling
or no prefill, and a second multi-token call, raise instead of attending over
the wrong positions. No GPU: the checks run before any kernel."""
import math

import pytest
import torch

from kvquant.hf_cache import KVQuantState, check_decode_call, check_prefill_call


def _state(filled: bool):
    st = KVQuantState(None, 2, 4, torch.ones(64))
    if filled:
        st.pk = [{}, {}]
        st.pv = [{}, {}]
    return st


def test_decode_accepts_the_default_call():
    st = _state(True)
    check_decode_call(st, 0, None, None)
    check_decode_call(st, 0, torch.ones(2, 1, 1, 9, dtype=torch.bool), 1 / math.sqrt(128))
    check_decode_call(st, 1, torch.zeros(2, 1, 1, 9), 1 / math.sqrt(128))


def test_decode_rejects_a_mask_that_hides_cached_positions():
    st = _state(True)
    m = torch.ones(2, 1, 1, 9, dtype=torch.bool)
    m[1, 0, 0, :3] = False  # left padding of the second sequence
    with pytest.raises(RuntimeError, match="hides cached positions"):
        check_decode_call(st, 0, m, None)
    add = torch.zeros(2, 1, 1, 9)
    add[0, 0, 0, 0] = torch.finfo(torch.float32).min
    with pytest.raises(RuntimeError, match="hides cached positions"):
        check_decode_call(st, 0, add, None)


def test_decode_rejects_another_scaling_and_a_missing_prefill():
    with pytest.raises(RuntimeError, match="scaling"):
        check_decode_call(_state(True), 0, None, 0.1)
    with pytest.raises(RuntimeError, match="before the prefill"):
        check_decode_call(_state(False), 0, None, None)


def test_second_prefill_is_rejected():
    check_prefill_call(_state(False), 0)
    with pytest.raises(RuntimeError, match="after the prefill"):
        check_prefill_call(_state(True), 1)
