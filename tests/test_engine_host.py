"""Host logic of the decode engine's device-error handling (CPU only).

A kernel that gives up a bounded wait records an error code instead of
hanging; the engine must raise after its next sync, clear the code and zero
the persistent step's counters before the next launch.  The failure is
injected on the host (a fake error word), never by a GPU fault.
"""
import types

import pytest
import torch

from spmv_decode_b200 import _lib
from spmv_decode_b200.engine import DecodeEngine


class _FakeLib:
    def __init__(self):
        self.resets = []

    def nms_step_reset(self, handle, stream):
        self.resets.append((handle, stream))
        return 0


def _fake_engine():
    return types.SimpleNamespace(_steps={False: "step-fixed", True: "step-adv"}, device=torch.device("cpu"),
                                 amax_counter=torch.ones(1, dtype=torch.int32))


def test_check_device_raises_clears_and_resets(monkeypatch):
    fake = _FakeLib()
    word = {"v": 3}

    def device_error(clear=True):
        v = word["v"]
        if clear:
            word["v"] = 0
        return v

    monkeypatch.setattr(_lib, "device_error", device_error)
    monkeypatch.setattr(_lib, "lib", lambda: fake)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda dev=None: types.SimpleNamespace(cuda_stream=77))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda dev=None: None)
    eng = _fake_engine()
    with pytest.raises(RuntimeError, match=r"error 3 \(grid barrier"):
        DecodeEngine.check_device(eng)
    assert word["v"] == 0
    assert sorted(fake.resets) == [("step-adv", 77), ("step-fixed", 77)]
    assert int(eng.amax_counter.item()) == 0  # the head's arrival counter starts clean too
    # Clean word: no exception, no reset.
    DecodeEngine.check_device(eng)
    assert len(fake.resets) == 2


def test_check_device_names_every_code(monkeypatch):
    from spmv_decode_b200.engine import DEVICE_ERRORS

    assert set(DEVICE_ERRORS) == {1, 2, 3, 4, 5, 6}
    monkeypatch.setattr(_lib, "lib", lambda: _FakeLib())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda dev=None: types.SimpleNamespace(cuda_stream=0))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda dev=None: None)
    for code, text in DEVICE_ERRORS.items():
        monkeypatch.setattr(_lib, "device_error", lambda clear=True, c=code: c)
        with pytest.raises(RuntimeError, match=text):
            DecodeEngine.check_device(_fake_engine())


def test_auto_executor_by_layer_bytes():
    """Mode "auto" runs small layers on the plan executor and large ones on
    the persistent step (the measured crossover sits between Llama-3.1-8B's
    218 MB and Qwen3-32B's 488 MB of GEMV weights per layer)."""
    from spmv_decode_b200.engine import AUTO_PLAN_BELOW_LAYER_BYTES, auto_executor

    assert auto_executor(15.7e6) == "plan"
    assert auto_executor(218e6) == "plan"
    assert auto_executor(488e6) == "persistent"
    assert auto_executor(AUTO_PLAN_BELOW_LAYER_BYTES - 1) == "plan"
    assert auto_executor(AUTO_PLAN_BELOW_LAYER_BYTES) == "persistent"
