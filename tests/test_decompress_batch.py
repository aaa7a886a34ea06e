"""compute_decompress_batch follows krunch/cpp_path.py:531-580 (A-21)."""
import types

import pytest

from krunch_b200 import codec


def _props(sms, major, mem):
    return types.SimpleNamespace(multi_processor_count=sms, major=major, total_memory=mem)


@pytest.fixture()
def fake_gpu(monkeypatch):
    def install(sms, major, mem):
        monkeypatch.setattr(codec.torch.cuda, "is_available", lambda: True)
        monkeypatch.setattr(codec.torch.cuda, "get_device_properties",
                            lambda d=0: _props(sms, major, mem))
    monkeypatch.delenv("KRUNCH_DECOMPRESS_BATCH", raising=False)
    return install


def test_b200_saturation(fake_gpu):
    fake_gpu(148, 10, 183359 << 20)
    assert codec.compute_decompress_batch() == 1184
    assert codec.compute_decompress_batch(300) == 300
    assert codec.compute_decompress_batch(5000) == 1184


@pytest.mark.parametrize("sms,major,mem,want", [
    (40, 7, 16 << 30, 80),        # T4: legacy path, SMs x 2
    (80, 8, 24 << 30, 640),       # A10G
    (132, 9, 80 << 30, 1056),     # H100
    (148, 10, 1 << 30, 546),      # memory cap: 0.8 GiB / 1.5 MiB
])
def test_reference_table(fake_gpu, sms, major, mem, want):
    fake_gpu(sms, major, mem)
    assert codec.compute_decompress_batch() == want


def test_env_override_and_no_gpu(monkeypatch):
    monkeypatch.setenv("KRUNCH_DECOMPRESS_BATCH", "48")
    assert codec.compute_decompress_batch() == 48
    assert codec.compute_decompress_batch(10) == 10
    monkeypatch.setenv("KRUNCH_DECOMPRESS_BATCH", "junk")
    monkeypatch.setattr(codec.torch.cuda, "is_available", lambda: False)
    assert codec.compute_decompress_batch() == 64
    assert codec.compute_decompress_batch(7) == 7
