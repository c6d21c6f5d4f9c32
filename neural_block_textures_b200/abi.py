"""ctypes binding of libntc_b200.so (include/ntc_b200.h).

The structures mirror the C description structs field for field; test_abi.py checks their layout
against the C++ compiler's view of include/ntc_cuda.h and the reference's cuda/ntc_cuda.h. Loading
fails loudly: there is no fallback implementation of any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

MAX_LEVELS = 3
MAX_POS = 16
MAX_OUT = 12
MAX_HIDDEN = 8
MAX_CH = 16
MAX_QES_CH = 64
MAX_DCT_CH = 4

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libntc_b200.so"


class LevelDesc(C.Structure):
    _fields_ = [("W", C.c_int), ("H", C.c_int), ("C", C.c_int), ("off", C.c_size_t), ("nearest", C.c_bool)]


class PosDesc(C.Structure):
    _fields_ = [("kind", C.c_int)]


class ModelDesc(C.Structure):
    _fields_ = [
        ("W", C.c_int), ("H", C.c_int), ("T", C.c_int),
        ("nlev", C.c_int), ("lv", LevelDesc * MAX_LEVELS),
        ("npos", C.c_int), ("pos", PosDesc * MAX_POS),
        ("nin", C.c_int), ("nout", C.c_int),
        ("nhidden", C.c_int), ("hidden", C.c_int * MAX_HIDDEN),
        ("leak", C.c_float),
        ("clamp_out", C.c_bool),
        ("cw", C.c_float * MAX_OUT),
        ("wsum", C.c_float),
        ("qat_bits", C.c_int * MAX_CH),
        ("qat", C.c_int),
        ("qat_grid", C.POINTER(C.c_float)),
        ("qes_bits", C.c_int * MAX_LEVELS),
        ("dct", C.c_int), ("dct_C", C.c_int), ("dct_N", C.c_int), ("dct_dc_step", C.c_int),
        ("dct_q", C.c_int * MAX_DCT_CH),
        ("dct_basis", C.POINTER(C.c_float)),
        ("dct_zigzag", C.POINTER(C.c_int)),
        ("max_pairs", C.c_int), ("max_batch", C.c_int),
        ("seed", C.c_uint64),
    ]


class QesDesc(C.Structure):
    _fields_ = [
        ("bits", C.c_int * MAX_LEVELS),
        ("live", C.c_int), ("frozen", C.c_int),
        ("lo", (C.c_float * MAX_QES_CH) * MAX_LEVELS),
        ("hi", (C.c_float * MAX_QES_CH) * MAX_LEVELS),
        ("range", (C.c_float * MAX_QES_CH) * MAX_LEVELS),
        ("grid_off", (C.c_int * MAX_QES_CH) * MAX_LEVELS),
    ]


class DctDesc(C.Structure):
    _fields_ = [
        ("live", C.c_int), ("C", C.c_int), ("BW", C.c_int), ("BH", C.c_int), ("N", C.c_int), ("dc_step", C.c_int),
        ("rate_es", C.c_int), ("rate_trunc", C.c_int), ("rate_scale", C.c_float), ("lam_t16", C.c_float * 16),
        ("lo_w16", C.c_int),
        ("deadzone", C.c_int),
    ]


class ContainerDesc(C.Structure):
    """ntcb_container_desc: a parsed .ntcb header."""
    _fields_ = [
        ("version", C.c_int), ("img_w", C.c_int), ("img_h", C.c_int), ("src_w", C.c_int), ("src_h", C.c_int),
        ("T", C.c_int), ("nlevels", C.c_int), ("nin", C.c_int), ("nout", C.c_int), ("nhidden", C.c_int),
        ("hidden", C.c_int * MAX_HIDDEN), ("leak", C.c_float), ("clamp_out", C.c_int),
        ("lv_W", C.c_int * MAX_LEVELS), ("lv_H", C.c_int * MAX_LEVELS), ("lv_C", C.c_int * MAX_LEVELS),
        ("lv_nearest", C.c_int * MAX_LEVELS), ("lv_mode", C.c_int * MAX_LEVELS), ("lv_bits", C.c_int * MAX_LEVELS),
        ("npos", C.c_int), ("pos_kind", C.c_int * MAX_POS),
        ("nz", C.c_longlong), ("nweights", C.c_longlong),
    ]


class ProgressStats(C.Structure):
    """ntcb_progress_stats: the progress print's figures (main.cpp:4155-4205)."""
    _fields_ = [
        ("mse", C.c_double), ("mse_tex", C.c_double * (MAX_OUT // 3)),
        ("mse_q", C.c_double), ("mse_q_tex", C.c_double * (MAX_OUT // 3)),
        ("bpp_fp32", C.c_double), ("bpp_q8", C.c_double), ("bpp_q8_ent", C.c_double), ("bpp_q8_ctx", C.c_double),
        ("bpp_ctx_level0", C.c_double), ("bpp_est", C.c_double), ("bits_mlp", C.c_double),
        ("bits_raw_latent", C.c_double), ("bits_header", C.c_double),
        ("lat_mean", C.c_float * MAX_LEVELS), ("lat_sd", C.c_float * MAX_LEVELS), ("lat_max", C.c_float * MAX_LEVELS),
        ("qat_off_grid", C.c_longlong),
        ("level0_dct", C.c_int),
        ("dct_bits_raw", C.c_double), ("dct_bits_h0", C.c_double), ("dct_bits_ctx", C.c_double), ("dct_bits_header", C.c_double),
    ]


_fp = C.POINTER(C.c_float)
_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)
_i16p = C.POINTER(C.c_int16)
_u8p = C.POINTER(C.c_uint8)
_i32p = C.POINTER(C.c_int32)
_vp = C.c_void_p

# name -> (restype, argtypes); the list is the ABI surface of include/ntc_b200.h.
SIGNATURES = {
    "ntcb_create": (_vp, []),
    "ntcb_destroy": (None, [_vp]),
    "ntcb_init": (C.c_int, [_vp, C.POINTER(ModelDesc), _fp, _fp, _fp, C.c_char_p, C.c_size_t]),
    "ntcb_banner": (C.c_size_t, [_vp, C.c_char_p, C.c_size_t]),
    "ntcb_upload_model": (None, [_vp, _fp, _fp]),
    "ntcb_download_model": (None, [_vp, _fp, _fp]),
    "ntcb_set_qes": (None, [_vp, C.POINTER(QesDesc), _fp, C.c_size_t]),
    "ntcb_snap_latent": (None, [_vp]),
    "ntcb_shadow_pull": (None, [_vp, C.c_size_t, C.c_size_t, C.c_float]),
    "ntcb_download_zq": (None, [_vp, _fp]),
    "ntcb_set_dct": (None, [_vp, C.POINTER(DctDesc), _u8p, _i16p, _ip]),
    "ntcb_download_dct": (None, [_vp, _i16p, _u8p]),
    "ntcb_download_dct_rate": (None, [_vp, _i32p, _i32p, _ip, _ip, _ip, _ip]),
    "ntcb_mlp_step": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int]),
    "ntcb_mlp_step_fd": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int]),
    "ntcb_reset_mlp_adam": (None, [_vp]),
    "ntcb_mlp_stats": (None, [_vp, _dp, _dp]),
    "ntcb_lat_step": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int]),
    "ntcb_qat_search": (None, [_vp]),
    "ntcb_decode_full": (None, [_vp, _fp, _fp]),
    "ntcb_debug_last_batch": (C.c_size_t, [_vp, _ip, C.c_size_t]),
    "ntcb_debug_last_dl": (C.c_size_t, [_vp, _dp, C.c_size_t]),
    "ntcb_debug_last_zgrad": (C.c_size_t, [_vp, _fp, C.c_size_t]),
    "ntcb_debug_last_fitness": (C.c_size_t, [_vp, _dp, _dp, C.c_size_t]),
    "ntcb_set_stream": (None, [_vp, _vp]),
    "ntcb_kernel_timing": (None, [_vp, C.c_int]),
    "ntcb_kernel_time": (None, [_vp, C.c_char_p, _dp, _ip]),
    "ntcb_kernel_timing_only": (None, [_vp, C.c_char_p]),
    "ntcb_launch_count": (C.c_longlong, [_vp]),
    "ntcb_set_pop_kernel": (None, [_vp, C.c_int]),
    "ntcb_dct_probe": (C.c_size_t, [_vp, C.POINTER(C.c_uint8), _fp, C.c_size_t]),
    "ntcb_cpp_dct_probe": (C.c_size_t, [_vp, C.POINTER(C.c_uint8), _fp, C.c_size_t]),
    "ntcb_print_stats": (C.c_int, [_vp, C.POINTER(C.c_int), C.c_int, C.c_int, _fp, C.POINTER(ProgressStats)]),
    "ntcb_cpp_print_stats": (C.c_int, [_vp, C.POINTER(C.c_int), C.c_int, C.c_int, _fp, C.POINTER(ProgressStats)]),
    "ntcb_container_info": (C.c_int, [_u8p, C.c_size_t, C.POINTER(ContainerDesc), C.c_char_p, C.c_size_t]),
    "ntcb_decoder_open": (_vp, [_u8p, C.c_size_t, C.c_char_p, C.c_size_t]),
    "ntcb_decoder_get_info": (None, [_vp, C.POINTER(ContainerDesc)]),
    "ntcb_decoder_model": (None, [_vp, _fp, _fp]),
    "ntcb_decoder_rgb8": (C.c_size_t, [_vp, C.c_int, C.c_int, _u8p, C.c_size_t]),
    "ntcb_decoder_rgb8_device": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "ntcb_decoder_close": (None, [_vp]),
    "ntcb_dct_tables": (None, [C.c_int, C.c_int, _fp, _ip, _ip]),
    "ntcb_pop_kernel": (C.c_int, [_vp]),
    "ntcb_fp32_peak_tflops": (C.c_double, []),
    "ntcb_footprint_ranges": (C.c_int, [C.c_int, C.c_int, C.c_int, _ip, _ip]),
    "ntcb_es_fitness_noalloc": (C.c_int, [C.POINTER(ModelDesc), C.c_int, C.c_float, C.c_int, C.c_int, _fp, _fp, _fp, C.c_int, _dp,
                                          C.c_char_p, C.c_size_t]),
    "ntcb_noise_fill": (None, [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_size_t, _fp, C.POINTER(C.c_uint32)]),
    "ntcb_shard_es_block_bytes": (C.c_longlong, [_vp, C.c_int, C.c_int, C.c_int]),
    "ntcb_shard_mlp_eval_grad": (None, [_vp, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "ntcb_shard_mlp_apply_grad": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, _vp, C.c_int]),
    "ntcb_shard_lat_plan": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(C.c_longlong)]),
    "ntcb_shard_lat_step_rows": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int, _vp]),
    "ntcb_shard_lat_install": (None, [_vp, C.c_int, _vp]),
    "ntcb_shard_fd_eval": (None, [_vp, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int, _vp]),
    "ntcb_shard_fd_apply": (None, [_vp, C.c_float, C.c_float, _vp]),
    "ntcb_shard_mlp_eval": (None, [_vp, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "ntcb_shard_mlp_apply": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, _vp]),
    "ntcb_shard_lat_eval": (None, [_vp, C.c_float, C.c_int, C.c_int, C.c_int, _vp]),
    "ntcb_shard_lat_apply": (None, [_vp, C.c_int, C.c_float, C.c_float, C.c_int, _vp, C.c_int]),
    "ntcb_shard_qat": (None, [_vp, C.c_int, C.c_int, _vp]),
    "ntcb_shard_qat_apply": (None, [_vp, _vp]),
    "ntcb_comm_unique_id": (C.c_int, [C.POINTER(C.c_ubyte), C.c_char_p, C.c_size_t]),
    "ntcb_comm_create": (_vp, [C.POINTER(C.c_ubyte), C.c_int, C.c_int, C.c_char_p, C.c_size_t]),
    "ntcb_comm_destroy": (None, [_vp]),
    "ntcb_nccl_version": (C.c_int, []),
    "ntcb_shard_iteration_plan": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _ip, _ip, C.c_char_p,
                                            C.c_size_t]),
    "ntcb_shard_iteration": (None, [_vp, _vp, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float,
                                    C.c_int]),
    "ntcb_p2p_export": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_ubyte), C.c_char_p, C.c_size_t]),
    "ntcb_p2p_import": (C.c_int, [_vp, C.POINTER(C.c_ubyte), C.c_int, C.c_int, C.c_char_p, C.c_size_t]),
    "ntcb_p2p_release": (None, [_vp]),
    "ntcb_p2p_set_poll_limit": (None, [_vp, C.c_uint]),
    "ntcb_p2p_barrier": (C.c_int, [_vp, C.c_uint]),
}

COMM_ID_BYTES = 128   # NTCB_COMM_ID_BYTES
P2P_HANDLE_BYTES = 64   # NTCB_P2P_HANDLE_BYTES

_lib = None


def load_library(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads the in-tree libntc_b200.so (built by neural_block_textures_b200.build). Raises if missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"libntc_b200.so not found at {p}: build it with `python -m neural_block_textures_b200.build`")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib
