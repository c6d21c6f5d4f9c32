"""The device .ntcb decoder (ntcb_decoder_*) against the oracle reader and the reference's own decoder output.

Bars: the reconstructed latent and the weights bit-identical to the oracle's reading of the file (grid indices
and DCT reconstruction are exact); RGB8 equal to the reference decoder's (ntc_decode --exact) except at most
0.1 % of the bytes, each by one level (a float within ~1e-5 of an 8-bit rounding edge; the decode itself agrees
with the oracle to 1e-5)."""
from pathlib import Path

import numpy as np
import pytest

from neural_block_textures_b200 import ntcb
from oracle import ntcb_oracle

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "ntcb"
CASES = ["qat_q8", "qes", "dct", "dct2_dz0", "material"]


def _data(name: str) -> bytes:
    return (FIX / f"{name}.ntcb").read_bytes()


@pytest.mark.parametrize("name", CASES)
def test_decoder_latent_and_weights_exact(name, cuda_device):
    data = _data(name)
    h, spec, z, p = ntcb_oracle.read(data)
    with ntcb.NtcbDecoder(data) as dec:
        dz, dw = dec.model()
    assert np.array_equal(dz.view(np.uint32), z.view(np.uint32))
    assert np.array_equal(dw.view(np.uint32), p.view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_decoder_rgb8_matches_reference_decoder(name, cuda_device):
    g = np.load(FIX / f"{name}.npz")["decoder_rgb8"]
    with ntcb.NtcbDecoder(_data(name)) as dec:
        rgb = dec.rgb8()
    assert rgb.shape == g.shape
    d = np.abs(rgb.astype(np.int32) - g)
    assert d.max() <= 1 and np.mean(d > 0) <= 1e-3, (int((d > 0).sum()), d.max())


def test_decoder_crop_and_device_output(cuda_device):
    import torch
    data = _data("dct")   # 60 x 52 source padded to 64 x 56
    with ntcb.NtcbDecoder(data) as dec:
        full = dec.rgb8(64, 56)
        src = dec.rgb8()
        assert src.shape == (1, 52, 60, 3) and np.array_equal(full[:, :52, :60], src)
        out = torch.zeros(3 * 64 * 56, dtype=torch.uint8, device="cuda")
        s = torch.cuda.Stream()
        dec.rgb8_device(out.data_ptr(), 64, 56, s.cuda_stream)
        s.synchronize()
        assert np.array_equal(out.cpu().numpy().reshape(1, 56, 64, 3), full)
        with pytest.raises(ntcb.NtcbError):
            dec.rgb8(65, 56)


def test_decoder_refuses_damaged_file(cuda_device):
    b = bytearray(_data("qes"))
    b[100] ^= 0xFF
    with pytest.raises(ntcb.NtcbError, match="hash"):
        ntcb.NtcbDecoder(bytes(b))
