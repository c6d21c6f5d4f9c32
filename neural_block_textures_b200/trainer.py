"""Python mirror of the reference backend's ntc_cuda::Trainer (cuda/ntc_cuda.h:78-132) over the C ABI.

Every method has the reference member's name and argument meaning and takes / returns host numpy
arrays; all work runs in libntc_b200.so on the current CUDA device. As in the reference, a runtime
failure inside the library prints a message and ends the process (the caller has no error path);
init() returns False plus a reason for a model the backend does not support.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import abi


def _fptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _ptr(a: np.ndarray | None, ctype):
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(ctype))


class Trainer:
    def __init__(self) -> None:
        self.lib = abi.load_library()
        self.h = self.lib.ntcb_create()
        self.nz = 0
        self.P = 0
        self.npix = 0
        self.nout = 0
        self._desc = None

    def close(self) -> None:
        if self.h:
            self.lib.ntcb_destroy(self.h)
            self.h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- Trainer::init (cuda/ntc_cuda.h:85)
    def init(self, desc: abi.ModelDesc, z: np.ndarray, p: np.ndarray, target: np.ndarray) -> tuple[bool, str]:
        why = C.create_string_buffer(512)
        self._desc = desc
        self.nz = int(z.size)
        self.P = int(p.size)
        self.npix = desc.W * desc.H
        self.nout = desc.nout
        assert target.size == self.npix * self.nout
        ok = self.lib.ntcb_init(self.h, C.byref(desc), _fptr(z), _fptr(p), _fptr(target), why, 512)
        return bool(ok), why.value.decode()

    def banner(self) -> str:
        buf = C.create_string_buffer(512)
        self.lib.ntcb_banner(self.h, buf, 512)
        return buf.value.decode()

    def upload_model(self, z: np.ndarray, p: np.ndarray) -> None:
        self.lib.ntcb_upload_model(self.h, _fptr(z), _fptr(p))

    def download_model(self, z: np.ndarray | None = None, p: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
        """The latent and the weights; into z / p when given (contiguous float32 of nz / P values, e.g. pinned host
        arrays reused every step), else into new arrays."""
        if z is None:
            z = np.empty(self.nz, np.float32)
        if p is None:
            p = np.empty(self.P, np.float32)
        for a, n in ((z, self.nz), (p, self.P)):
            if a.dtype != np.float32 or a.size != n or not a.flags["C_CONTIGUOUS"]:
                raise ValueError(f"download_model: output must be a contiguous float32 array of {n} values")
        self.lib.ntcb_download_model(self.h, _fptr(z), _fptr(p))
        return z, p

    def set_qes(self, q: abi.QesDesc, grid: np.ndarray) -> None:
        self.lib.ntcb_set_qes(self.h, C.byref(q), _fptr(grid), grid.size)

    def snap_latent(self) -> None:
        self.lib.ntcb_snap_latent(self.h)

    def shadow_pull(self, off: int, n: int, f: float) -> None:
        self.lib.ntcb_shadow_pull(self.h, off, n, f)

    def download_zq(self) -> np.ndarray:
        z = np.empty(self.nz, np.float32)
        self.lib.ntcb_download_zq(self.h, _fptr(z))
        return z

    def set_dct(self, d: abi.DctDesc, code: np.ndarray, sym: np.ndarray, step: np.ndarray) -> None:
        self.lib.ntcb_set_dct(self.h, C.byref(d), _ptr(code, C.c_uint8), _ptr(sym, C.c_int16), _ptr(step, C.c_int))

    def download_dct(self, n_blocks_channels: int) -> tuple[np.ndarray, np.ndarray]:
        sym = np.empty(n_blocks_channels * 64, np.int16)
        code = np.empty(n_blocks_channels, np.uint8)
        self.lib.ntcb_download_dct(self.h, _ptr(sym, C.c_int16), _ptr(code, C.c_uint8))
        return sym, code

    def download_dct_rate(self, n_blocks_channels: int) -> dict:
        bits = np.empty(n_blocks_channels, np.int32)
        dbl = np.empty(n_blocks_channels, np.int32)
        v = [C.c_int() for _ in range(4)]
        self.lib.ntcb_download_dct_rate(self.h, _ptr(bits, C.c_int32), _ptr(dbl, C.c_int32), *[C.byref(x) for x in v])
        return {"bits": bits, "dbits_last_pair": dbl, "ntrunc": v[0].value, "nz_before": v[1].value,
                "hits": v[2].value, "evals": v[3].value}

    # ---- steps
    def mlp_step(self, it: int, sigma: float, lr: float, N: int, M: int) -> None:
        self.lib.ntcb_mlp_step(self.h, it, sigma, lr, N, M)

    def mlp_step_fd(self, it: int, h: float, lr: float, M: int) -> None:
        self.lib.ntcb_mlp_step_fd(self.h, it, h, lr, M)

    def reset_mlp_adam(self) -> None:
        self.lib.ntcb_reset_mlp_adam(self.h)

    def mlp_stats(self) -> tuple[float, float]:
        a, b = C.c_double(), C.c_double()
        self.lib.ntcb_mlp_stats(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def lat_step(self, it: int, sigma: float, lr: float, K: int) -> None:
        self.lib.ntcb_lat_step(self.h, it, sigma, lr, K)

    def qat_search(self) -> None:
        self.lib.ntcb_qat_search(self.h)

    def decode_full(self, z_host: np.ndarray | None = None) -> np.ndarray:
        img = np.empty(self.npix * self.nout, np.float32)
        self.lib.ntcb_decode_full(self.h, _fptr(z_host), _fptr(img))
        return img

    # ---- verification helpers
    def debug_last_batch(self) -> np.ndarray:
        n = self.lib.ntcb_debug_last_batch(self.h, None, 0)
        out = np.empty(n, np.int32)
        self.lib.ntcb_debug_last_batch(self.h, _ptr(out, C.c_int), n)
        return out

    def debug_last_dl(self) -> np.ndarray:
        n = self.lib.ntcb_debug_last_dl(self.h, None, 0)
        out = np.empty(n, np.float64)
        self.lib.ntcb_debug_last_dl(self.h, _ptr(out, C.c_double), n)
        return out

    def debug_last_zgrad(self) -> np.ndarray:
        out = np.empty(self.nz, np.float32)
        self.lib.ntcb_debug_last_zgrad(self.h, _fptr(out), self.nz)
        return out

    def debug_last_fitness(self) -> tuple[np.ndarray, np.ndarray]:
        n = self.lib.ntcb_debug_last_fitness(self.h, None, None, 0)
        lp = np.empty(n, np.float64)
        lm = np.empty(n, np.float64)
        self.lib.ntcb_debug_last_fitness(self.h, _ptr(lp, C.c_double), _ptr(lm, C.c_double), n)
        return lp, lm

    # ---- additions
    def set_stream(self, stream_handle: int | None) -> None:
        self.lib.ntcb_set_stream(self.h, C.c_void_p(stream_handle) if stream_handle else None)

    def kernel_timing(self, enable: bool) -> None:
        self.lib.ntcb_kernel_timing(self.h, 1 if enable else 0)

    def kernel_timing_only(self, kernel: str | None) -> None:
        """Time only this kernel class while timing is on (None: every class)."""
        self.lib.ntcb_kernel_timing_only(self.h, kernel.encode() if kernel else None)

    def kernel_time(self, kernel: str) -> tuple[float, int]:
        ms, n = C.c_double(), C.c_int()
        self.lib.ntcb_kernel_time(self.h, kernel.encode(), C.byref(ms), C.byref(n))
        return ms.value, n.value

    def launch_count(self) -> int:
        return int(self.lib.ntcb_launch_count(self.h))

    def dct_probe(self) -> tuple[np.ndarray, np.ndarray]:
        """Device DCT sensitivity probe: (codes uint8, gains float32), [block raster][level-0 channel]."""
        n = self.lib.ntcb_dct_probe(self.h, None, None, 0)
        codes = np.zeros(n, np.uint8)
        gains = np.zeros(n, np.float32)
        self.lib.ntcb_dct_probe(self.h, codes.ctypes.data_as(C.POINTER(C.c_uint8)), _ptr(gains, C.c_float), n)
        return codes, gains

    def print_stats(self, level_bits=None, eval_w: int = 0, eval_h: int = 0, want_zq: bool = False):
        """The progress print's statistics on the device (ntcb_print_stats): (ProgressStats, zq or None).
        level_bits: post-hoc depth per level (default 8, the reference's --qbits)."""
        lb = np.full(abi.MAX_LEVELS, 8, np.int32)
        if level_bits is not None:
            lb[: len(level_bits)] = level_bits
        out = abi.ProgressStats()
        zq = np.empty(self.nz, np.float32) if want_zq else None
        rc = self.lib.ntcb_print_stats(self.h, _ptr(lb, C.c_int), eval_w, eval_h, _fptr(zq), C.byref(out))
        if rc != 0:
            raise ValueError("ntcb_print_stats: a post-hoc depth outside 1..16")
        return out, zq

    def set_pop_kernel(self, tensor: bool) -> None:
        """True: ES pairs on the tensor-core (3xTF32) kernel; False: the bit-exact packed-FP32 kernel."""
        self.lib.ntcb_set_pop_kernel(self.h, 1 if tensor else 0)

    def pop_kernel(self) -> str:
        return "tensor" if self.lib.ntcb_pop_kernel(self.h) else "ffma"

    def shard_mlp_eval(self, it: int, sigma: float, N: int, M: int, p0: int, p1: int, fit_dev) -> None:
        """fit_dev: a CUDA tensor (or device pointer) of 2 * (p1 - p0) doubles on this trainer's GPU."""
        ptr = fit_dev if isinstance(fit_dev, int) else fit_dev.data_ptr()
        self.lib.ntcb_shard_mlp_eval(self.h, it, sigma, N, M, p0, p1, C.c_void_p(ptr))

    def shard_mlp_apply(self, it: int, sigma: float, lr: float, N: int, M: int, fit_all_dev) -> None:
        """fit_all_dev: a CUDA tensor (or device pointer) with all N pairs' (L+, L-) in pair order."""
        ptr = fit_all_dev if isinstance(fit_all_dev, int) else fit_all_dev.data_ptr()
        self.lib.ntcb_shard_mlp_apply(self.h, it, sigma, lr, N, M, C.c_void_p(ptr))

    def shard_es_block_bytes(self, N: int, p0: int, p1: int) -> int:
        return int(self.lib.ntcb_shard_es_block_bytes(self.h, N, p0, p1))

    def shard_mlp_eval_grad(self, it: int, sigma: float, N: int, M: int, p0: int, p1: int, block_dev) -> None:
        """block_dev: device buffer of shard_es_block_bytes(N, p0, p1) bytes (fitness, then gradient segments)."""
        self.lib.ntcb_shard_mlp_eval_grad(self.h, it, sigma, N, M, p0, p1, C.c_void_p(_dptr(block_dev)))

    def shard_mlp_apply_grad(self, it: int, sigma: float, lr: float, N: int, M: int, blocks_dev, world: int) -> None:
        self.lib.ntcb_shard_mlp_apply_grad(self.h, it, sigma, lr, N, M, C.c_void_p(_dptr(blocks_dev)), world)

    def shard_lat_plan(self, world: int, rank: int):
        """(level, ta, tb, pa, pb, n) of the texel-row latent sharding, or None when it does not apply."""
        plan = (C.c_longlong * 6)()
        if not self.lib.ntcb_shard_lat_plan(self.h, world, rank, plan):
            return None
        return tuple(int(v) for v in plan)

    def shard_lat_step_rows(self, it: int, sigma: float, lr: float, K: int, world: int, rank: int, zblock_dev) -> None:
        self.lib.ntcb_shard_lat_step_rows(self.h, it, sigma, lr, K, world, rank, C.c_void_p(_dptr(zblock_dev)))

    def shard_lat_install(self, level: int, level_dev) -> None:
        self.lib.ntcb_shard_lat_install(self.h, level, C.c_void_p(_dptr(level_dev)))

    def shard_fd_eval(self, it: int, h: float, M: int, j_begin: int, j_end: int, fit_dev) -> None:
        """fit_dev: device buffer of >= 2 * (j_end - j_begin) doubles; receives (L+, L-) of weights [j_begin, j_end)."""
        self.lib.ntcb_shard_fd_eval(self.h, it, h, M, j_begin, j_end, C.c_void_p(_dptr(fit_dev)))

    def shard_fd_apply(self, h: float, lr: float, fit_all_dev) -> None:
        """fit_all_dev: device buffer whose first 2 * P doubles are every weight's (L+, L-) in weight order."""
        self.lib.ntcb_shard_fd_apply(self.h, h, lr, C.c_void_p(_dptr(fit_all_dev)))

    def shard_lat_eval(self, sigma: float, K: int, row_begin: int, row_end: int, block_dev) -> None:
        """block_dev: a CUDA tensor of K * (row_end - row_begin) * W float32, laid out [K][rows * W]."""
        self.lib.ntcb_shard_lat_eval(self.h, sigma, K, row_begin, row_end, C.c_void_p(_dptr(block_dev)))

    def shard_lat_apply(self, it: int, sigma: float, lr: float, K: int, blocks_dev, rows_per_block: int) -> None:
        """blocks_dev: every rank's block in row order, each [K][rows_per_block * W]."""
        self.lib.ntcb_shard_lat_apply(self.h, it, sigma, lr, K, C.c_void_p(_dptr(blocks_dev)), rows_per_block)

    def shard_qat(self, trow_begin: int, trow_end: int, level0_dev) -> None:
        """level0_dev: a CUDA tensor of the level-0 W * H * C floats; the searched rows are written into it."""
        self.lib.ntcb_shard_qat(self.h, trow_begin, trow_end, C.c_void_p(_dptr(level0_dev)))

    def shard_qat_apply(self, level0_all_dev) -> None:
        self.lib.ntcb_shard_qat_apply(self.h, C.c_void_p(_dptr(level0_all_dev)))

    # ---- native sharded iteration (addition): one call per iteration, the library's own NCCL communicator
    def shard_iteration_plan(self, world: int, rank: int, mlp_mode: int, N: int, M: int, K: int, qat: bool):
        """(ok, mlp_exchange, lat_exchange, reason) of ntcb_shard_iteration for this model (include/ntc_b200.h)."""
        mx, lx = C.c_int(0), C.c_int(0)
        why = C.create_string_buffer(256)
        ok = self.lib.ntcb_shard_iteration_plan(self.h, world, rank, mlp_mode, N, M, K, int(qat), C.byref(mx), C.byref(lx), why, 256)
        return bool(ok), mx.value, lx.value, why.value.decode()

    def shard_iteration(self, comm: "Comm", it: int, mlp_mode: int, mlp_sigma: float, mlp_lr: float, N: int, M: int, K: int,
                        lat_sigma: float, lat_lr: float, qat: bool) -> None:
        self.lib.ntcb_shard_iteration(self.h, comm.h, it, mlp_mode, mlp_sigma, mlp_lr, N, M, K, lat_sigma, lat_lr, int(qat))


    def p2p_export(self, world: int, rank: int, N: int, K: int, qat: bool) -> bytes:
        """Allocates this rank's peer-exchange buffer and returns its IPC handle (ntcb_p2p_export)."""
        h = (C.c_ubyte * abi.P2P_HANDLE_BYTES)()
        why = C.create_string_buffer(256)
        if not self.lib.ntcb_p2p_export(self.h, world, rank, N, K, int(qat), h, why, 256):
            raise RuntimeError("ntcb_p2p_export: " + why.value.decode())
        return bytes(h)

    def p2p_import(self, handles: bytes, world: int, rank: int) -> None:
        """Maps every peer's exchange buffer (handles of all ranks in rank order, ntcb_p2p_import)."""
        if len(handles) != world * abi.P2P_HANDLE_BYTES:
            raise ValueError("need one handle per rank")
        buf = (C.c_ubyte * len(handles)).from_buffer_copy(handles)
        why = C.create_string_buffer(256)
        if not self.lib.ntcb_p2p_import(self.h, buf, world, rank, why, 256):
            raise RuntimeError("ntcb_p2p_import: " + why.value.decode())


    def p2p_set_poll_limit(self, polls: int) -> None:
        """Polls of one staged peer line before an exchange wait fails (0: the default; ntcb_p2p_set_poll_limit)."""
        self.lib.ntcb_p2p_set_poll_limit(self.h, polls)

    def p2p_barrier(self, polls: int = 0) -> int:
        """Peer barrier through the exchange buffers (ntcb_p2p_barrier): 0 when every peer arrived, 2 when a wait ran
        out (the error word is returned and cleared instead of exiting)."""
        return int(self.lib.ntcb_p2p_barrier(self.h, polls))

    def p2p_release(self) -> None:
        """Unmaps the peers' exchange buffers (ntcb_p2p_release); every rank, then a barrier, before destroying."""
        self.lib.ntcb_p2p_release(self.h)


class Comm:
    """The library's NCCL communicator (ntcb_comm_*): `uid` is the id rank 0 made with Comm.unique_id(), handed to
    every rank; create it with the rank's device current."""

    def __init__(self, uid: bytes, world: int, rank: int) -> None:
        self.lib = abi.load_library()
        if len(uid) != abi.COMM_ID_BYTES:
            raise ValueError("NCCL unique id must be %d bytes" % abi.COMM_ID_BYTES)
        why = C.create_string_buffer(256)
        buf = (C.c_ubyte * abi.COMM_ID_BYTES).from_buffer_copy(uid)
        self.h = self.lib.ntcb_comm_create(buf, world, rank, why, 256)
        if not self.h:
            raise RuntimeError("ntcb_comm_create: " + why.value.decode())
        self.world, self.rank = world, rank

    @staticmethod
    def unique_id() -> bytes:
        lib = abi.load_library()
        buf = (C.c_ubyte * abi.COMM_ID_BYTES)()
        why = C.create_string_buffer(256)
        if not lib.ntcb_comm_unique_id(buf, why, 256):
            raise RuntimeError("ntcb_comm_unique_id: " + why.value.decode())
        return bytes(buf)

    def close(self) -> None:
        if self.h:
            self.lib.ntcb_comm_destroy(self.h)
            self.h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def _dptr(x) -> int:
    return x if isinstance(x, int) else x.data_ptr()

