"""Host-side mirror of gemma4.kt's floattensor layer, backed by libg4b200.

Reference interface (lib/src/main/kotlin/io/github/lbenedetto/internal/):
  GGMLType            gguf/GGMLType.kt:12-80      -> GGMLType
  FloatTensorFactory  floattensor/FloatTensorFactory.kt:7-23 -> FloatTensorFactory.create
  FloatTensor.matmul  floattensor/FloatTensor.kt:18-29       -> CudaFloatTensor.matmul
  FloatTensor.get     (per type)                              -> CudaFloatTensor.dequant

Activations ("that"/"out") may be torch CUDA tensors (device path, stream
ordered) or numpy float32 arrays (host path: the Kotlin heap FloatArray case,
synchronous).  Errors mirror the reference: UnsupportedOperationException ->
UnsupportedOperation, IllegalArgumentException -> ValueError.
"""
from __future__ import annotations

import ctypes as C
from enum import IntEnum

import numpy as np

from ._lib import G4Error, check, lib

QK_K = 256  # GGMLType.kt:5


class UnsupportedOperation(G4Error):
    """UnsupportedOperationException (FloatTensorFactory.kt:21, GGMLType.kt:77)."""


class GGMLType(IntEnum):
    """GGML tensor types FloatTensorFactory.create accepts (FloatTensorFactory.kt:7-23,
    GGMLType.kt:16-55)."""

    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_1 = 7
    Q8_0 = 8
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    BF16 = 30
    MXFP4 = 39

    @property
    def block_size(self) -> int:
        return {GGMLType.Q4_0: 32, GGMLType.Q4_1: 32, GGMLType.Q5_1: 32, GGMLType.Q8_0: 32, GGMLType.MXFP4: 32,
                GGMLType.Q4_K: QK_K, GGMLType.Q5_K: QK_K, GGMLType.Q6_K: QK_K}.get(self, 1)

    @property
    def type_size(self) -> int:
        return {GGMLType.F32: 4, GGMLType.F16: 2, GGMLType.BF16: 2, GGMLType.Q4_0: 18, GGMLType.Q4_1: 20,
                GGMLType.Q5_1: 24, GGMLType.Q8_0: 34, GGMLType.Q4_K: 144, GGMLType.Q5_K: 176, GGMLType.Q6_K: 210,
                GGMLType.MXFP4: 17}[self]

    def byte_size_for(self, n_elems: int) -> int:
        """GGMLType.byteSizeFor (GGMLType.kt:58-62)."""
        t = n_elems * self.type_size
        if t % self.block_size:
            raise ValueError(f"{n_elems} elements are not a whole number of {self.name} blocks")
        return t // self.block_size

    @staticmethod
    def from_id(type_id: int) -> "GGMLType":
        try:
            return GGMLType(type_id)
        except ValueError:
            raise UnsupportedOperation(f"Quantization format {type_id}") from None


def _is_torch(a) -> bool:
    return type(a).__module__.startswith("torch")


def _stream_ptr(stream) -> int:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return int(stream)


def row_shard(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Output rows [begin, begin + count) that `rank` of `world` owns when a
    [rows, cols] tensor is split by output rows (one contiguous slice per GPU,
    rank order = row order, so an all-gather of the slices is y)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if rows % world:
        raise ValueError(f"{rows} rows do not split evenly over {world} GPUs")
    per = rows // world
    return rank * per, per


class Context:
    """One g4_ctx per CUDA device (per process / host thread)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        rc = lib().g4_init(device, C.byref(h))
        if rc != 0:
            msg = lib().g4_last_error(None)
            raise G4Error(f"g4_init({device}) failed: {msg.decode() if msg else rc}")
        self.handle = h
        self.device = device

    def close(self) -> None:
        if self.handle:
            lib().g4_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self, stream=None) -> None:
        check(lib().g4_sync(self.handle, C.c_void_p(_stream_ptr(stream))), self.handle, "g4_sync")

    def last_error(self) -> str:
        m = lib().g4_last_error(self.handle)
        return m.decode() if m else ""

    @staticmethod
    def dist_unique_id() -> bytes:
        """A fresh NCCL unique id (G4_NCCL_ID_BYTES) for rank 0 to share."""
        uid = (C.c_ubyte * 128)()
        rc = lib().g4_dist_unique_id(uid)
        if rc != 0:
            raise G4Error(f"g4_dist_unique_id failed ({rc})")
        return bytes(uid)

    def dist_init(self, rank: int, world: int, uid: bytes, timeout_ms: int | None = None) -> None:
        """Join the NCCL communicator of `world` GPUs (one Context per GPU).
        Waits on peers are bounded by timeout_ms (default: G4_DIST_TIMEOUT_MS
        or 120 s); on expiry the communicator is aborted and G4Error raised."""
        if len(uid) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        buf = (C.c_ubyte * 128).from_buffer_copy(uid)
        if timeout_ms is None:
            rc = lib().g4_dist_init(self.handle, rank, world, buf)
        else:
            rc = lib().g4_dist_init_timeout(self.handle, rank, world, buf, int(timeout_ms))
        check(rc, self.handle, "g4_dist_init")

    def dist_abort(self) -> None:
        """Abort this context's communicator (single-GPU calls keep working)."""
        check(lib().g4_dist_abort(self.handle), self.handle, "g4_dist_abort")


class CudaFloatTensor:
    """A weight tensor resident in HBM in its GGUF block layout.

    Stand-in for Q8_0FloatTensor / Q4_KFloatTensor / Q6_KFloatTensor /
    BF16FloatTensor / F32FloatTensor: same `size`, `matmul` and element
    semantics, with the dot products computed by the sm_100a kernels.
    """

    def __init__(self, ctx: Context, handle: C.c_void_p, ggml_type: GGMLType, size: int):
        self.ctx = ctx
        self.handle = handle
        self.ggml_type = ggml_type
        self.size = size

    def free(self) -> None:
        if self.handle:
            lib().g4_tensor_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def device_ptr(self) -> int:
        return lib().g4_tensor_device_ptr(self.handle) or 0

    @property
    def nbytes(self) -> int:
        return int(lib().g4_tensor_nbytes(self.handle))

    def matmul(self, that, out, dim0: int, dim1: int, this_offset: int = 0, stream=None) -> None:
        """FloatTensor.matmul(that, out, dim0, dim1[, thisOffset]) (FloatTensor.kt:18-29):
        out[i] = dot(this_offset + i*dim1, that, 0, dim1) for i < dim0."""
        if dim0 < 0 or dim1 < 0 or this_offset < 0:
            raise ValueError("negative matmul dimension")
        if _is_torch(that):
            if not (that.is_cuda and out.is_cuda):
                raise ValueError("torch activations must be CUDA tensors")
            if that.numel() < dim1 or out.numel() < dim0:
                raise ValueError("activation buffers too small")
            rc = lib().g4_matmul(self.ctx.handle, self.handle, this_offset, C.c_void_p(that.data_ptr()),
                                 C.c_void_p(out.data_ptr()), dim0, dim1, C.c_void_p(_stream_ptr(stream)))
            check(rc, self.ctx.handle, "g4_matmul")
        else:
            x = np.ascontiguousarray(that, dtype=np.float32)
            if not (isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous):
                raise ValueError("host output must be a contiguous float32 numpy array")
            if x.size < dim1 or out.size < dim0:
                raise ValueError("activation buffers too small")
            rc = lib().g4_matmul_host(self.ctx.handle, self.handle, this_offset, x.ctypes.data_as(C.c_void_p),
                                      out.ctypes.data_as(C.c_void_p), dim0, dim1)
            check(rc, self.ctx.handle, "g4_matmul_host")

    def matmul_sharded(self, that, out, rows: int, cols: int, stream=None) -> None:
        """matmul of a row-sharded tensor (this holds rows row_shard(rows, world, rank)):
        computes the local slice of out and all-gathers the full out[rows] on
        every rank.  that/out are CUDA tensors; out holds all rows."""
        if not (_is_torch(that) and _is_torch(out) and that.is_cuda and out.is_cuda):
            raise ValueError("matmul_sharded takes CUDA tensors")
        if that.numel() < cols or out.numel() < rows:
            raise ValueError("activation buffers too small")
        rc = lib().g4_matmul_sharded(self.ctx.handle, self.handle, C.c_void_p(that.data_ptr()),
                                     C.c_void_p(out.data_ptr()), rows, cols, C.c_void_p(_stream_ptr(stream)))
        check(rc, self.ctx.handle, "g4_matmul_sharded")

    def dequant(self, offset: int, n: int, out=None, stream=None):
        """[get(offset + i) for i < n] (the per-type FloatTensor.get), on the GPU."""
        import torch

        if out is None:
            out = torch.empty(n, dtype=torch.float32, device=f"cuda:{self.ctx.device}")
        rc = lib().g4_dequant(self.ctx.handle, self.handle, offset, n, C.c_void_p(out.data_ptr()),
                              C.c_void_p(_stream_ptr(stream)))
        check(rc, self.ctx.handle, "g4_dequant")
        return out


class FloatTensorFactory:
    """FloatTensorFactory.create (FloatTensorFactory.kt:7-23) for device tensors."""

    @staticmethod
    def create(ctx: Context, ggml_type, raw, n_elems: int) -> CudaFloatTensor:
        t = GGMLType.from_id(int(ggml_type))
        buf = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray)
                                   else raw.view(np.uint8).reshape(-1))
        h = C.c_void_p()
        rc = lib().g4_tensor_upload(ctx.handle, int(t), buf.ctypes.data_as(C.c_void_p), buf.nbytes, n_elems,
                                    C.byref(h))
        if rc == -2:
            raise UnsupportedOperation(ctx.last_error())
        if rc == -1:
            raise ValueError(ctx.last_error())
        check(rc, ctx.handle, "g4_tensor_upload")
        return CudaFloatTensor(ctx, h, t, n_elems)

    @staticmethod
    def create_rows(ctx: Context, ggml_type, raw, cols: int, row_begin: int, row_count: int) -> CudaFloatTensor:
        """Upload one output-row shard of a [rows, cols] tensor."""
        t = GGMLType.from_id(int(ggml_type))
        buf = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray)
                                   else raw.view(np.uint8).reshape(-1))
        h = C.c_void_p()
        rc = lib().g4_tensor_upload_rows(ctx.handle, int(t), buf.ctypes.data_as(C.c_void_p), cols, row_begin,
                                         row_count, C.byref(h))
        if rc == -1:
            raise ValueError(ctx.last_error())
        check(rc, ctx.handle, "g4_tensor_upload_rows")
        return CudaFloatTensor(ctx, h, t, row_count * cols)
