"""Streaming input (int_crush_converter_b200.tensor_io): the safetensors reader
against safetensors' own loader, byte for byte, and the lazy calibration
loader against torch.load.  The GPU test reads straight into device memory."""

import os

import pytest
import torch

from int_crush_converter_b200 import tensor_io as TI


def _write(tmp):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(3)
    sd = {
        "double_blocks.0.img_mlp.0.weight": (torch.randn(96, 64, generator=g) * 0.02).half(),
        "double_blocks.0.img_mlp.0.bias": torch.randn(96, generator=g).bfloat16(),
        "x.codes": torch.randint(-8, 8, (7, 33), generator=g, dtype=torch.int8),
        "x.empty": torch.zeros(0, 5),
        "x.f32": torch.randn(3, 5, 7, generator=g),
    }
    p = os.path.join(tmp, "m.safetensors")
    save_file(sd, p, metadata={"format": "pt", "int_crush.rot_size": "256"})
    return p, sd


def test_reader_matches_safetensors(tmp_path):
    p, sd = _write(str(tmp_path))
    r = TI.SafetensorsReader(p, chunk_bytes=1000)  # several chunks per tensor
    assert sorted(r) == sorted(sd) and len(r) == len(sd)
    assert r.metadata["int_crush.rot_size"] == "256"
    for k, v in sd.items():
        t = r[k]
        assert t.dtype == v.dtype and t.shape == v.shape
        assert torch.equal(t.view(torch.uint8) if t.numel() else t, v.view(torch.uint8) if v.numel() else v)
    r.close()


def test_lazy_calibration(tmp_path):
    g = torch.Generator().manual_seed(4)
    cal = {"hessians": {"a": torch.randn(16, 16, generator=g), "b": torch.randn(8, 8, generator=g)},
           "amax_per_channel": {"a": torch.rand(16, generator=g)}, "metadata": {"num_samples": 128}}
    p = os.path.join(str(tmp_path), "cal.pt")
    torch.save(cal, p)
    lz = TI.load_calibration_lazy(p)
    assert lz["metadata"] == {"num_samples": 128}
    assert torch.equal(lz["hessians"]["a"], cal["hessians"]["a"])
    assert torch.equal(lz["amax_per_channel"]["a"], cal["amax_per_channel"]["a"])


@pytest.mark.gpu
def test_reader_to_device(tmp_path):
    p, sd = _write(str(tmp_path))
    r = TI.SafetensorsReader(p, chunk_bytes=1000)
    for k, v in sd.items():
        t = r.get(k, "cuda")
        assert t.is_cuda and t.dtype == v.dtype and t.shape == v.shape
        assert torch.equal(t.cpu(), v)
