"""The .ntcb container (the reference trainer's --write-ntcb output) decoded on the device, through the C ABI
(ntcb_container_info, ntcb_decoder_*).

    info = container_info(data)                    # host-only parse and validation, no GPU
    with NtcbDecoder(data) as dec:                 # upload + latent reconstruction on the current GPU
        rgb = dec.rgb8()                           # [T][src_h][src_w][3] uint8, as the reference writes its PNGs
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import abi

MODE_NAMES = {0: "q8", 1: "qes", 2: "qat", 3: "dct"}


class NtcbError(ValueError):
    """The container was refused; the message names the first problem."""


def _buf(data: bytes | np.ndarray):
    a = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else np.ascontiguousarray(data, np.uint8)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint8))


def container_info(data: bytes | np.ndarray) -> abi.ContainerDesc:
    """Parses and validates a container on the host; raises NtcbError with the reason on refusal."""
    lib = abi.load_library()
    a, p = _buf(data)
    info = abi.ContainerDesc()
    err = C.create_string_buffer(512)
    if lib.ntcb_container_info(p, a.size, C.byref(info), err, 512) != 0:
        raise NtcbError(err.value.decode())
    return info


def dct_tables(q: int, dc_step: int):
    """(basis [64] float32, zigzag [64] int32, steps [16][64] int32) as the decoder builds them."""
    lib = abi.load_library()
    b = np.zeros(64, np.float32); z = np.zeros(64, np.int32); s = np.zeros(16 * 64, np.int32)
    lib.ntcb_dct_tables(q, dc_step, b.ctypes.data_as(C.POINTER(C.c_float)), z.ctypes.data_as(C.POINTER(C.c_int)),
                        s.ctypes.data_as(C.POINTER(C.c_int)))
    return b, z, s.reshape(16, 64)


class NtcbDecoder:
    """One container resident on the current CUDA device."""

    def __init__(self, data: bytes | np.ndarray):
        self.lib = abi.load_library()
        a, p = _buf(data)
        err = C.create_string_buffer(512)
        self.h = self.lib.ntcb_decoder_open(p, a.size, err, 512)
        if not self.h:
            raise NtcbError(err.value.decode())
        self.info = abi.ContainerDesc()
        self.lib.ntcb_decoder_get_info(self.h, C.byref(self.info))

    def model(self) -> tuple[np.ndarray, np.ndarray]:
        """The reconstructed latent (flat, levels in order) and the weights (the fp16 values as float32)."""
        z = np.zeros(self.info.nz, np.float32)
        w = np.zeros(self.info.nweights, np.float32)
        self.lib.ntcb_decoder_model(self.h, z.ctypes.data_as(C.POINTER(C.c_float)), w.ctypes.data_as(C.POINTER(C.c_float)))
        return z, w

    def rgb8(self, crop_w: int = 0, crop_h: int = 0) -> np.ndarray:
        """[T][crop_h][crop_w][3] uint8 (0 = the source size)."""
        n = self.lib.ntcb_decoder_rgb8(self.h, crop_w, crop_h, None, 0)
        if n == 0:
            raise NtcbError("crop larger than the decode size")
        out = np.zeros(n, np.uint8)
        self.lib.ntcb_decoder_rgb8(self.h, crop_w, crop_h, out.ctypes.data_as(C.POINTER(C.c_uint8)), n)
        cw = crop_w or self.info.src_w
        ch = crop_h or self.info.src_h
        return out.reshape(self.info.T, ch, cw, 3)

    def rgb8_device(self, out_ptr: int, crop_w: int = 0, crop_h: int = 0, stream: int = 0) -> None:
        """Decode into device memory at out_ptr on `stream` (0 = the decoder's own), without synchronising."""
        if self.lib.ntcb_decoder_rgb8_device(self.h, crop_w, crop_h, C.c_void_p(out_ptr), C.c_void_p(stream or None)) != 0:
            raise NtcbError("crop larger than the decode size")

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.ntcb_decoder_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
