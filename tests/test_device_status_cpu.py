"""The product path reads the per-device status word: a kernel that skipped a
row or gave up a pipeline wait must stop the decode, not let it carry on with
incomplete K/V or attention output.  Checked on the CPU by faking the status
through the C ABI (fdl_last_device_error) -- no kernel runs."""
import ctypes

import pytest
import torch

from fast_v2_b200 import _lib
from fast_v2_b200.block_decode import BlockDiffusionDecoder, BlockDiffusionLM, Geometry

TINY = Geometry(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=128, ffn=128, vocab=300)


class _FakeAbi:
    """Stands in for libfdl_b200.so: fdl_last_device_error reports `code` once,
    then 0 (the real call clears the word on read)."""

    def __init__(self, code, info=7):
        self.code, self.info, self.calls = code, info, 0

    def fdl_last_device_error(self, code_ref, info_ref):
        self.calls += 1
        code_ref._obj.value = self.code
        info_ref._obj.value = self.info
        self.code = 0
        return 0


@pytest.fixture
def fake_abi(monkeypatch):
    def install(code, info=7):
        fake = _FakeAbi(code, info)
        monkeypatch.setattr(_lib, "abi", lambda: fake)
        return fake

    return install


def test_check_device_raises_on_every_nonzero_code(fake_abi):
    for code in (1, 2, 3):
        fake_abi(code, info=11)
        with pytest.raises(_lib.DeviceError) as e:
            _lib.check_device("unit")
        assert e.value.code == code and e.value.info == 11
        assert "unit" in str(e.value)
    fake_abi(0)
    _lib.check_device("unit")  # ok: no raise


def test_timeout_name_is_in_the_message(fake_abi):
    fake_abi(3)
    with pytest.raises(_lib.DeviceError, match="FDL_DEV_TIMEOUT"):
        _lib.check_device("decode")


def _cpu_decoder(monkeypatch):
    model = BlockDiffusionLM(TINY, device="cpu", dtype=torch.float32, load_ops=False)
    dec = BlockDiffusionDecoder(model, batch=2, prompt_len=32, gen_len=32, mask_id=299, stop_id=298, pad_id=297)
    # No kernels on the CPU: every step is a no-op that leaves the status
    # buffer at "no mask left", so the block loop runs one step and commits.
    monkeypatch.setattr(dec, "_run", lambda key: None)
    return dec


def test_decode_block_raises_when_a_kernel_recorded_an_error(monkeypatch, fake_abi):
    dec = _cpu_decoder(monkeypatch)
    fake = fake_abi(3)
    with pytest.raises(_lib.DeviceError, match="decode_block"):
        dec.decode_block(torch.zeros(2, 1, dtype=torch.long))
    assert fake.calls == 1


def test_decode_block_passes_with_a_clean_status(monkeypatch, fake_abi):
    dec = _cpu_decoder(monkeypatch)
    fake = fake_abi(0)
    x, nxt = dec.decode_block(torch.zeros(2, 1, dtype=torch.long))
    assert x.shape == (2, 32) and nxt.shape == (2, 1)
    assert fake.calls == 1


def test_real_library_status_call_signature():
    # The real entry point's ctypes signature: two out-pointers, int return.
    lib = _lib.abi()
    f = lib.fdl_last_device_error
    assert f.restype == ctypes.c_int32
    assert f.argtypes == [ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)]
