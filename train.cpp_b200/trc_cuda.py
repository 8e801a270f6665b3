"""Python host mirror of train.cpp's quantized-weight hot path on the B200 (libtrc_cuda.so).

The functions keep the reference's names and argument meaning (paths relative to the train.cpp
source tree):

  gguf_tensor_to_f32(type, blocks)        src/io/trc_gguf.cpp:966-1049 (Q* branch :1040-1044)
  gguf_load_tensor(type, host_blocks, dst) src/io/trc_gguf.cpp:1051-1094 (F32 destination)
  mul_mat(a, b)                            src/ops/trc_ops.cpp:366-385 + trc_cpu_ops.cpp:182-216
  mul_mat_q(type, w_blocks, ...)           fused dequant + mul_mat (no reference counterpart:
                                           the reference must materialise the F32 weight)
  cont / acc / repeat_back / repeat / add / sub / mul / div / sum
                                           src/backends/cpu/trc_cpu_ops.cpp (compute_dup :219,
                                           compute_acc :954, compute_repeat_back :932, ...)

Tensors are torch CUDA tensors used purely as device memory. A ggml tensor with
ne = [ne0, ne1, ne2, ne3] is a torch tensor of shape (ne3, ne2, ne1, ne0); any torch stride
pattern maps to ggml byte strides nb (so `t.transpose(-1, -2)` is ggml's `transpose`).
Every call goes through the C ABI of include/trc_cuda.h; there is no CPU fallback: if the
library is missing or a call fails, TrcCudaError is raised, mirroring the reference's TRC_ABORT.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Sequence

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libtrc_cuda.so"

# ggml type ids (include/traincpp/trc_types.h:11-49)
TYPE_F32, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q5_0, TYPE_Q5_1, TYPE_Q8_0 = 0, 2, 3, 6, 7, 8
TYPE_NAMES = {TYPE_Q4_0: "q4_0", TYPE_Q4_1: "q4_1", TYPE_Q5_0: "q5_0", TYPE_Q5_1: "q5_1", TYPE_Q8_0: "q8_0"}
BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q4_1: 20, TYPE_Q5_0: 22, TYPE_Q5_1: 24, TYPE_Q8_0: 34}
QK = 32  # weights per block

MM_ACCUMULATE, MM_SIMT, MM_ONE_CTA, MM_NO_PRETAIL, MM_FUSED, MM_TWO_STEP = 1, 2, 4, 8, 16, 32
BIN_ADD, BIN_SUB, BIN_MUL, BIN_DIV = 0, 1, 2, 3


class TrcCudaError(RuntimeError):
    pass


class View(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_int64 * 4)]


class DequantJob(ctypes.Structure):
    _fields_ = [("blocks", ctypes.c_void_p), ("out", ctypes.c_void_p), ("n_blocks", ctypes.c_int64),
                ("type", ctypes.c_int32), ("reserved", ctypes.c_int32)]


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libtrc_cuda.so (built in-tree by build.py). Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise TrcCudaError(f"{LIB_PATH} is missing: run train.cpp_b200/build.py (no CPU fallback exists)")
    L = ctypes.CDLL(str(LIB_PATH))
    P, I, I64, U32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_size_t
    VP = ctypes.POINTER(View)
    sig = {
        "trc_cuda_abi_version": (I, []),
        "trc_cuda_status_string": (ctypes.c_char_p, [I]),
        "trc_cuda_last_cuda_error": (I, []),
        "trc_cuda_device_error": (I, [ctypes.POINTER(I), I]),
        "trc_cuda_launch_count": (ctypes.c_uint64, []),
        "trc_cuda_sm_count": (I, []),
        "trc_cuda_block_bytes": (SZ, [I]),
        "trc_cuda_dequant": (I, [I, P, I64, P, P]),
        "trc_cuda_dequant_many": (I, [ctypes.POINTER(DequantJob), I, P]),
        "trc_cuda_load_quant": (I, [I, P, I64, P, P, P]),
        "trc_cuda_load_quant_static": (I, [I, P, I64, P, P]),
        "trc_cuda_mul_mat": (I, [VP, VP, VP, U32, P]),
        "trc_cuda_mul_mat_q": (I, [I, P, I64, I64, I, VP, VP, U32, P]),
        "trc_cuda_mul_mat_kernel": (I, [VP, VP, VP, U32]),
        "trc_cuda_mul_mat_repeat_back": (I, [VP, VP, VP, U32, P]),
        "trc_cuda_cont": (I, [VP, VP, P]),
        "trc_cuda_acc": (I, [P, I64, VP, I64, I64, I64, I64, P]),
        "trc_cuda_repeat_back": (I, [VP, VP, P]),
        "trc_cuda_repeat": (I, [VP, VP, P]),
        "trc_cuda_binary": (I, [I, VP, VP, VP, P]),
        "trc_cuda_sum_workspace_bytes": (SZ, [I64]),
        "trc_cuda_sum": (I, [VP, P, P, SZ, P]),
        "trc_cuda_fill": (I, [P, I64, ctypes.c_float, P]),
        "trc_cuda_dequant_many_to_peers": (I, [ctypes.POINTER(DequantJob), I, P, ctypes.POINTER(P), I, P]),
        "trc_cuda_rt_malloc": (I, [ctypes.POINTER(P), SZ]),
        "trc_cuda_rt_free": (I, [P]),
        "trc_cuda_rt_ipc_get_handle": (I, [P, P]),
        "trc_cuda_rt_ipc_open": (I, [P, ctypes.POINTER(P)]),
        "trc_cuda_rt_ipc_close": (I, [P]),
        "trc_cuda_rt_can_access_peer": (I, [I, I, ctypes.POINTER(I)]),
        "trc_cuda_unary": (I, [I, VP, VP, ctypes.c_float, P]),
        "trc_cuda_selftest_wait_timeout": (I, [ctypes.c_uint64, ctypes.POINTER(I)]),
        "trc_cuda_stream_probe": (I, [P, P, I64, I, P]),
        "trc_cuda_stream_probe_bulk": (I, [P, P, I64, I, P]),
        "trc_cuda_tf32_mma_probe": (I, [I, I, P]),
        "trc_cuda_sum_rows": (I, [VP, VP, I, P]),
        "trc_cuda_opt_step_adamw": (I, [P, P, P, P, I64, P, P]),
        "trc_cuda_opt_step_sgd": (I, [P, P, P, I64, P, P]),
        "trc_cuda_sum_sqr_workspace_bytes": (SZ, [I64]),
        "trc_cuda_sum_sqr_acc": (I, [P, P, I64, P, SZ, P]),
        "trc_cuda_clip_scale_inplace": (I, [P, I64, P, ctypes.c_float, ctypes.c_float, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.trc_cuda_status_string(status).decode()
        cuda_err = L.trc_cuda_last_cuda_error()
        raise TrcCudaError(f"{what}: {msg} (status {status}, cudaError {cuda_err})")


def _stream(stream: torch.cuda.Stream | None = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


# ------------------------------------------------------------------ ggml <-> torch views

def ggml_ne(t: torch.Tensor) -> list[int]:
    shape = list(t.shape)[::-1]
    if len(shape) > 4:
        raise TrcCudaError("ggml tensors have at most 4 dimensions")
    return shape + [1] * (4 - len(shape))


def view_of(t: torch.Tensor) -> View:
    """ggml view (ne, byte strides nb) of a float32 CUDA tensor with any strides."""
    if t.dtype != torch.float32:
        raise TrcCudaError(f"expected float32, got {t.dtype}")
    if not t.is_cuda:
        raise TrcCudaError("expected a CUDA tensor (device memory)")
    ne = ggml_ne(t)
    st = [s * 4 for s in list(t.stride())[::-1]]
    nb = st + [0] * (4 - len(st))
    # strides of padded size-1 dimensions: the contiguous value, as ggml sets them
    for d in range(len(st), 4):
        nb[d] = nb[d - 1] * ne[d - 1] if d > 0 else 4
    v = View()
    v.data = t.data_ptr()
    for i in range(4):
        v.ne[i] = ne[i]
        v.nb[i] = nb[i]
    return v


def ggml_empty(ne: Sequence[int], device="cuda") -> torch.Tensor:
    """Contiguous F32 tensor with ggml extents ne (ne0 innermost)."""
    ne = list(ne) + [1] * (4 - len(ne))
    return torch.empty(ne[::-1], dtype=torch.float32, device=device)


def transpose(t: torch.Tensor) -> torch.Tensor:
    """ggml transpose = permute(1, 0, 2, 3): swaps ne0/ne1 (a strided view, no copy)."""
    return t.transpose(-1, -2)


# ------------------------------------------------------------------ dequantization

def block_bytes(qtype: int) -> int:
    return int(lib().trc_cuda_block_bytes(qtype))


def _check_f32_dst(dst: torch.Tensor, what: str, n_weights: int | None = None) -> None:
    """The kernels write 32 floats per block at dst.data_ptr(): dst must be a contiguous float32
    CUDA tensor of whole blocks (and of n_weights elements when that is given)."""
    if dst.dtype != torch.float32:
        raise TrcCudaError(f"{what}: destination must be float32, got {dst.dtype}")
    if not dst.is_cuda:
        raise TrcCudaError(f"{what}: destination must be a CUDA tensor (device memory)")
    if not dst.is_contiguous():
        raise TrcCudaError(f"{what}: destination must be contiguous")
    if dst.numel() % QK != 0:
        raise TrcCudaError(f"{what}: {dst.numel()} weights are not a whole number of 32-weight blocks")
    if n_weights is not None and dst.numel() < n_weights:
        raise TrcCudaError(f"{what}: destination holds {dst.numel()} floats, the tensor has {n_weights}")


def gguf_tensor_to_f32(qtype: int, blocks: torch.Tensor, n_elems: int | None = None,
                       out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Device dequantization of packed legacy blocks (uint8 CUDA tensor) to F32, bit-exact with the
    reference's host dequantizers. Returns a flat float32 tensor of 32 * n_blocks weights."""
    bb = block_bytes(qtype)
    if bb == 0:
        raise TrcCudaError(f"type {qtype} is not a legacy quantized type")
    if blocks.dtype != torch.uint8 or not blocks.is_cuda or not blocks.is_contiguous():
        raise TrcCudaError("blocks must be a contiguous uint8 CUDA tensor")
    n_blocks = blocks.numel() // bb
    if n_elems is not None:
        if n_elems % QK != 0:
            raise TrcCudaError(f"{n_elems} weights are not a whole number of 32-weight blocks")
        n_blocks = n_elems // QK
    if n_blocks * bb > blocks.numel():
        raise TrcCudaError("packed buffer is smaller than the tensor")
    if out is None:
        out = torch.empty(n_blocks * QK, dtype=torch.float32, device=blocks.device)
    _check_f32_dst(out, "gguf_tensor_to_f32", n_blocks * QK)
    _check(lib().trc_cuda_dequant(qtype, blocks.data_ptr(), n_blocks, out.data_ptr(), _stream(stream)),
           "trc_cuda_dequant")
    return out


class DequantBatch:
    """A prepared batch of dequant jobs (qtype, packed uint8 CUDA tensor, F32 output): the job
    array is built and checked once, and each call is one trc_cuda_dequant_many (one kernel
    launch per 256 jobs) with no per-job host work -- what a model loader replays per step."""

    def __init__(self, jobs: Sequence[tuple[int, torch.Tensor, torch.Tensor]]):
        self._keep = [(b, o) for _, b, o in jobs]  # the tensors must outlive the array
        self._arr = (DequantJob * max(1, len(jobs)))()
        self._n = len(jobs)
        for i, (qtype, blocks, out) in enumerate(jobs):
            bb = block_bytes(qtype)
            if bb == 0:
                raise TrcCudaError(f"type {qtype} is not a legacy quantized type")
            self._arr[i].blocks = blocks.data_ptr()
            self._arr[i].out = out.data_ptr()
            self._arr[i].n_blocks = out.numel() // QK
            self._arr[i].type = qtype
            if blocks.numel() < self._arr[i].n_blocks * bb:
                raise TrcCudaError("packed buffer is smaller than its output")

    def __len__(self) -> int:
        return self._n

    def __call__(self, stream=None) -> None:
        _check(lib().trc_cuda_dequant_many(self._arr, self._n, _stream(stream)), "trc_cuda_dequant_many")


def dequantize_many(jobs: Sequence[tuple[int, torch.Tensor, torch.Tensor]], stream=None) -> None:
    """Batched device dequantization: jobs of (qtype, packed uint8 CUDA tensor, F32 output)."""
    DequantBatch(jobs)(stream)


IPC_HANDLE_BYTES = 64


class _DeviceArray:
    """__cuda_array_interface__ over raw device memory, so torch.as_tensor can wrap it."""

    def __init__(self, ptr: int, shape, typestr: str, owner):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None, "stream": None}
        self._owner = owner


class PeerBuffer:
    """One device buffer per rank of a process group (one process per GPU on one node), each
    mapped into every other rank's address space with CUDA IPC: `bases[r]` is rank r's buffer as
    this process addresses it (plain peer loads and stores over NVLink; no multicast object).
    Allocated with trc_cuda_rt_malloc so that the IPC handle covers exactly this buffer.
    Collective: every rank of `group` constructs it with the same nbytes, and calls close()."""

    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist

        L = lib()
        self.nbytes = int(nbytes)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        ptr = ctypes.c_void_p()
        _check(L.trc_cuda_rt_malloc(ctypes.byref(ptr), self.nbytes), "trc_cuda_rt_malloc")
        self.ptr = ptr.value
        self._opened: list[int] = []
        handle = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
        _check(L.trc_cuda_rt_ipc_get_handle(ctypes.c_void_p(self.ptr), handle), "trc_cuda_rt_ipc_get_handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.ptr)
                continue
            raw = (ctypes.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(h)
            peer = ctypes.c_void_p()
            _check(L.trc_cuda_rt_ipc_open(raw, ctypes.byref(peer)), "trc_cuda_rt_ipc_open")
            self.bases.append(peer.value)
            self._opened.append(peer.value)

    def tensor(self, dtype=torch.float32) -> torch.Tensor:
        """The local buffer as a flat torch CUDA tensor (no copy; valid until close())."""
        item = torch.empty((), dtype=dtype).element_size()
        typestr = {torch.float32: "<f4", torch.uint8: "|u1", torch.int32: "<i4"}[dtype]
        return torch.as_tensor(_DeviceArray(self.ptr, (self.nbytes // item,), typestr, self),
                               device=f"cuda:{torch.cuda.current_device()}")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this one. Call after a barrier, when no rank still
        writes into another's buffer."""
        if self.ptr is None:
            return
        L = lib()
        for p in self._opened:
            L.trc_cuda_rt_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        L.trc_cuda_rt_free(ctypes.c_void_p(self.ptr))
        self.ptr = None


def dequantize_to_peers(jobs: Sequence[tuple[int, torch.Tensor, torch.Tensor]], buf: PeerBuffer,
                        stream=None) -> None:
    """Dequantize jobs whose F32 outputs lie in buf's local buffer and write every output at the
    same offset of every other rank's buffer as well (trc_cuda_dequant_many_to_peers): the
    all-gather of a row-sharded tensor fused into its dequantization, one launch per rank."""
    arr = (DequantJob * max(1, len(jobs)))()
    for i, (qtype, blocks, out) in enumerate(jobs):
        bb = block_bytes(qtype)
        arr[i].blocks = blocks.data_ptr()
        arr[i].out = out.data_ptr()
        arr[i].n_blocks = out.numel() // QK
        arr[i].type = qtype
        if blocks.numel() < arr[i].n_blocks * bb:
            raise TrcCudaError("packed buffer is smaller than its output")
        if not (buf.ptr <= out.data_ptr() and out.data_ptr() + out.numel() * 4 <= buf.ptr + buf.nbytes):
            raise TrcCudaError("dequantize_to_peers: an output lies outside the peer buffer")
    peers = [b for r, b in enumerate(buf.bases) if r != buf.rank]
    parr = (ctypes.c_void_p * max(1, len(peers)))(*peers)
    _check(lib().trc_cuda_dequant_many_to_peers(arr, len(jobs), ctypes.c_void_p(buf.ptr), parr, len(peers),
                                                _stream(stream)), "trc_cuda_dequant_many_to_peers")


def _host_bytes(host_blocks) -> tuple[int, int]:
    """Address and size of packed blocks in HOST memory (a contiguous CPU tensor or numpy array)."""
    if isinstance(host_blocks, torch.Tensor):
        if host_blocks.is_cuda or not host_blocks.is_contiguous():
            raise TrcCudaError("packed blocks must be a contiguous tensor in host memory")
        return host_blocks.data_ptr(), host_blocks.numel() * host_blocks.element_size()
    if not host_blocks.flags["C_CONTIGUOUS"]:
        raise TrcCudaError("packed blocks must be a contiguous array")
    return host_blocks.ctypes.data, host_blocks.nbytes


def gguf_load_tensor(qtype: int, host_blocks, dst: torch.Tensor, staging: torch.Tensor, stream=None) -> None:
    """Device-side gguf_load_tensor for a quantized file tensor and an F32 destination: uploads the
    packed HOST bytes (numpy array or CPU tensor, pinned for an asynchronous copy) into `staging`
    and dequantizes into `dst`."""
    ptr, nbytes = _host_bytes(host_blocks)
    _check_f32_dst(dst, "gguf_load_tensor")
    if staging.dtype != torch.uint8 or not staging.is_cuda or not staging.is_contiguous():
        raise TrcCudaError("gguf_load_tensor: staging must be a contiguous uint8 CUDA tensor")
    if block_bytes(qtype) == 0:
        raise TrcCudaError(f"gguf_load_tensor: type {qtype} is not a legacy quantized type")
    n_blocks = dst.numel() // QK
    if nbytes < n_blocks * block_bytes(qtype) or staging.numel() < n_blocks * block_bytes(qtype):
        raise TrcCudaError("host or staging buffer smaller than the tensor")
    _check(lib().trc_cuda_load_quant(qtype, ctypes.c_void_p(ptr), n_blocks, staging.data_ptr(), dst.data_ptr(),
                                     _stream(stream)), "trc_cuda_load_quant")


STATIC_STAGING_BYTES = 64 << 20
ETOOBIG = -6


def gguf_load_tensor_static(qtype: int, host_blocks, dst: torch.Tensor, stream=None) -> None:
    """gguf_load_tensor without a staging buffer and without any allocation: the packed bytes are
    staged in the library's fixed 64 MiB device array (for callers that cannot allocate device
    memory). Tensors larger than that are rejected; calls overlapping on the GPU race on the array."""
    ptr, nbytes = _host_bytes(host_blocks)
    _check_f32_dst(dst, "gguf_load_tensor_static")
    if block_bytes(qtype) == 0:
        raise TrcCudaError(f"gguf_load_tensor_static: type {qtype} is not a legacy quantized type")
    n_blocks = dst.numel() // QK
    if nbytes < n_blocks * block_bytes(qtype):
        raise TrcCudaError("host buffer smaller than the tensor")
    _check(lib().trc_cuda_load_quant_static(qtype, ctypes.c_void_p(ptr), n_blocks, dst.data_ptr(), _stream(stream)),
           "trc_cuda_load_quant_static")


# ------------------------------------------------------------------ mul_mat

def mul_mat_out_ne(a: torch.Tensor, b: torch.Tensor) -> list[int]:
    na, nb_ = ggml_ne(a), ggml_ne(b)
    return [na[1], nb_[1], nb_[2], nb_[3]]


def _mm_flags(accumulate: bool, simt: bool, one_cta: bool, no_pretail: bool = False, fused: bool = False,
              two_step: bool = False) -> int:
    return ((MM_ACCUMULATE if accumulate else 0) | (MM_SIMT if simt else 0) | (MM_ONE_CTA if one_cta else 0) |
            (MM_NO_PRETAIL if no_pretail else 0) | (MM_FUSED if fused else 0) | (MM_TWO_STEP if two_step else 0))


def mul_mat(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False,
            simt: bool = False, stream=None, one_cta: bool = False, no_pretail: bool = False) -> torch.Tensor:
    """ggml mul_mat: out[i, j, i2, i3] = sum_k a[k, i, i2 % a2, i3 % a3] * b[k, j, i2, i3]."""
    na, nb_ = ggml_ne(a), ggml_ne(b)
    if na[0] != nb_[0]:
        raise TrcCudaError(f"mul_mat: inner dims differ (a.ne0={na[0]}, b.ne0={nb_[0]})")
    if nb_[2] % na[2] or nb_[3] % na[3]:
        raise TrcCudaError("mul_mat: a's planes do not broadcast onto b's (b.ne % a.ne must be 0)")
    if out is None:
        out = ggml_empty(mul_mat_out_ne(a, b), device=a.device)
    flags = _mm_flags(accumulate, simt, one_cta, no_pretail)
    va, vb, vd = view_of(a), view_of(b), view_of(out)
    _check(lib().trc_cuda_mul_mat(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vd), flags, _stream(stream)),
           "trc_cuda_mul_mat")
    return out


def mul_mat_repeat_back(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, accumulate: bool = False,
                        simt: bool = False, stream=None, one_cta: bool = False,
                        no_pretail: bool = False) -> torch.Tensor:
    """out (+)= repeat_back(mul_mat(a, b), shape of out): the broadcast-plane reduction of the
    composed backward's dA fused into the GEMM (out may have fewer planes than b)."""
    flags = _mm_flags(accumulate, simt, one_cta, no_pretail)
    va, vb, vd = view_of(a), view_of(b), view_of(out)
    _check(lib().trc_cuda_mul_mat_repeat_back(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vd), flags,
                                              _stream(stream)), "trc_cuda_mul_mat_repeat_back")
    return out


KERNEL_TCGEN05, KERNEL_SIMT = 1, 2


def mul_mat_kernel(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, simt: bool = False) -> int:
    """Which kernel mul_mat would run for these views: KERNEL_TCGEN05 or KERNEL_SIMT."""
    va, vb, vd = view_of(a), view_of(b), view_of(out)
    r = lib().trc_cuda_mul_mat_kernel(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vd), MM_SIMT if simt else 0)
    if r < 0:
        _check(r, "trc_cuda_mul_mat_kernel")
    return r


def mul_mat_q(qtype: int, w_blocks: torch.Tensor, w_ne0: int, w_ne1: int, b: torch.Tensor,
              transposed: bool = False, out: torch.Tensor | None = None, accumulate: bool = False,
              stream=None, one_cta: bool = False, no_pretail: bool = False, fused: bool = False,
              simt: bool = False, two_step: bool = False) -> torch.Tensor:
    """dequant + mul_mat with a = W (transposed=False) or a = transpose(W), W being the frozen
    quantized weight of ggml shape [w_ne0, w_ne1] held as packed blocks on the device. The default
    is the fused dequant-in-prologue kernel (no copy of W) wherever it can stage the packed bytes
    by TMA, else, from 1024 columns of b on, W dequantized into scratch + the F32 kernel.
    fused=True / two_step=True force one of the two (same results). simt=True: dequant + the SIMT
    kernel, bit-exact with the reference."""
    K, M = (w_ne1, w_ne0) if transposed else (w_ne0, w_ne1)
    nb_ = ggml_ne(b)
    if nb_[0] != K:
        raise TrcCudaError(f"mul_mat_q: inner dims differ ({K} vs {nb_[0]})")
    if out is None:
        out = ggml_empty([M, nb_[1], nb_[2], nb_[3]], device=b.device)
    vb, vd = view_of(b), view_of(out)
    _check(lib().trc_cuda_mul_mat_q(qtype, w_blocks.data_ptr(), w_ne0, w_ne1, 1 if transposed else 0,
                                    ctypes.byref(vb), ctypes.byref(vd),
                                    _mm_flags(accumulate, simt, one_cta, no_pretail, fused, two_step),
                                    _stream(stream)), "trc_cuda_mul_mat_q")
    return out


# ------------------------------------------------------------------ graph ops

def cont(src: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    if out is None:
        out = ggml_empty(ggml_ne(src), device=src.device)
    vs, vd = view_of(src), view_of(out)
    _check(lib().trc_cuda_cont(ctypes.byref(vs), ctypes.byref(vd), _stream(stream)), "trc_cuda_cont")
    return out


def acc_(dst: torch.Tensor, b: torch.Tensor, nb1: int, nb2: int, nb3: int, offset: int, stream=None) -> torch.Tensor:
    """In-place acc (inplace=1): dst's bytes [offset + i0*4 + i1*nb1 + i2*nb2 + i3*nb3] += b."""
    if not dst.is_contiguous():
        raise TrcCudaError("acc: destination must be contiguous")
    vb = view_of(b)
    _check(lib().trc_cuda_acc(dst.data_ptr(), dst.numel() * 4, ctypes.byref(vb), nb1, nb2, nb3, offset,
                              _stream(stream)), "trc_cuda_acc")
    return dst


def repeat_back(src: torch.Tensor, dst_ne: Sequence[int], out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    if out is None:
        out = ggml_empty(dst_ne, device=src.device)
    vs, vd = view_of(src), view_of(out)
    _check(lib().trc_cuda_repeat_back(ctypes.byref(vs), ctypes.byref(vd), _stream(stream)), "trc_cuda_repeat_back")
    return out


def repeat(src: torch.Tensor, dst_ne: Sequence[int], out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    if out is None:
        out = ggml_empty(dst_ne, device=src.device)
    vs, vd = view_of(src), view_of(out)
    _check(lib().trc_cuda_repeat(ctypes.byref(vs), ctypes.byref(vd), _stream(stream)), "trc_cuda_repeat")
    return out


def _binary(op: int, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None, stream) -> torch.Tensor:
    if out is None:
        out = ggml_empty(ggml_ne(a), device=a.device)
    va, vb, vd = view_of(a), view_of(b), view_of(out)
    _check(lib().trc_cuda_binary(op, ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vd), _stream(stream)),
           "trc_cuda_binary")
    return out


def add(a, b, out=None, stream=None):
    return _binary(BIN_ADD, a, b, out, stream)


def sub(a, b, out=None, stream=None):
    return _binary(BIN_SUB, a, b, out, stream)


def mul(a, b, out=None, stream=None):
    return _binary(BIN_MUL, a, b, out, stream)


def div(a, b, out=None, stream=None):
    return _binary(BIN_DIV, a, b, out, stream)


def sum_workspace_bytes(n: int) -> int:
    return int(lib().trc_cuda_sum_workspace_bytes(n))


def sum(src: torch.Tensor, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
        stream=None) -> torch.Tensor:  # noqa: A001 (mirrors the reference op name)
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=src.device)
    need = sum_workspace_bytes(src.numel())
    if workspace is None:
        workspace = torch.empty((need + 7) // 8, dtype=torch.float64, device=src.device)
    vs = view_of(src)
    _check(lib().trc_cuda_sum(ctypes.byref(vs), out.data_ptr(), workspace.data_ptr(), workspace.numel() * 8,
                              _stream(stream)), "trc_cuda_sum")
    return out


def fill_(dst: torch.Tensor, value: float, stream=None) -> torch.Tensor:
    if not dst.is_contiguous() or dst.dtype != torch.float32:
        raise TrcCudaError("fill: destination must be a contiguous float32 tensor")
    _check(lib().trc_cuda_fill(dst.data_ptr(), dst.numel(), float(value), _stream(stream)), "trc_cuda_fill")
    return dst


# ------------------------------------------------------------------ diagnostics

def device_error(reset: bool = True) -> int:
    """Device error word of the current device: 0, or the code of a kernel that gave up a wait."""
    code = ctypes.c_int(0)
    _check(lib().trc_cuda_device_error(ctypes.byref(code), 1 if reset else 0), "trc_cuda_device_error")
    return code.value


def stream_probe(src: torch.Tensor, dst: torch.Tensor, ratio: int, stream=None, bulk: bool = False) -> None:
    """Streams src (read once) into ratio x its bytes of dst: the dequant's traffic mix, no math.
    bulk=True writes through shared memory and bulk copies, the dequant kernel's store path."""
    n16 = (src.numel() * src.element_size()) // 16 // (256 if bulk else 32) * (256 if bulk else 32)
    if dst.numel() * dst.element_size() < ratio * n16 * 16:
        raise TrcCudaError("stream_probe: destination too small")
    fn = lib().trc_cuda_stream_probe_bulk if bulk else lib().trc_cuda_stream_probe
    _check(fn(src.data_ptr(), dst.data_ptr(), n16, ratio, _stream(stream)), "trc_cuda_stream_probe")


def tf32_mma_probe(cta_group: int, iters: int, stream=None) -> float:
    """Launches the tcgen05 kind::tf32 ceiling probe; returns the FLOPs the launch executes (every
    MMA counted: divide by 3 for the 3xTF32 rate with F32 FLOPs counted once)."""
    _check(lib().trc_cuda_tf32_mma_probe(cta_group, iters, _stream(stream)), "trc_cuda_tf32_mma_probe")
    ctas = sm_count() if cta_group == 1 else 2 * (sm_count() // 2)
    return float(iters) * 6 * 2 * 128 * 256 * 8 * ctas


def selftest_wait_timeout(limit_ns: int) -> bool:
    """Runs the bounded-wait self-test; True when the wait ran out (the kernel returned on its own)."""
    done = ctypes.c_int(-1)
    _check(lib().trc_cuda_selftest_wait_timeout(limit_ns, ctypes.byref(done)), "trc_cuda_selftest_wait_timeout")
    return done.value == 0


def launch_count() -> int:
    return int(lib().trc_cuda_launch_count())


def sm_count() -> int:
    return int(lib().trc_cuda_sm_count())


def exported_symbols() -> list[str]:
    """Names of the functions declared in include/trc_cuda.h and include/trc_cuda_runtime.h
    (parsed), used by the CPU symbol test."""
    import re
    names: list[str] = []
    for hdr in ("trc_cuda.h", "trc_cuda_runtime.h"):
        text = (PKG.parent / "include" / hdr).read_text()
        names += re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(trc_cuda_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


if os.environ.get("TRC_CUDA_PRELOAD") == "1":  # opt-in eager load (used by smoke checks)
    lib()


# ------------------------------------------------------------------ the rest of a training step

UNARY_SQR, UNARY_SQRT, UNARY_ABS, UNARY_NEG, UNARY_SGN, UNARY_STEP, UNARY_SCALE = range(7)


def unary(op: int, src: torch.Tensor, out: torch.Tensor | None = None, param: float = 0.0,
          stream=None) -> torch.Tensor:
    """sqr / sqrt / abs / neg / sgn / step / scale(param), element by element (any strides)."""
    if out is None:
        out = ggml_empty(ggml_ne(src), device=src.device)
    vs, vd = view_of(src), view_of(out)
    _check(lib().trc_cuda_unary(op, ctypes.byref(vs), ctypes.byref(vd), param, _stream(stream)), "trc_cuda_unary")
    return out


def sqr(src: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    return unary(UNARY_SQR, src, out, 0.0, stream)


def scale(src: torch.Tensor, s: float, out=None, stream=None) -> torch.Tensor:
    return unary(UNARY_SCALE, src, out, s, stream)


def sum_rows(src: torch.Tensor, out: torch.Tensor | None = None, mean: bool = False, stream=None) -> torch.Tensor:
    """ggml sum_rows (or mean): one value per row, summed in double in index order."""
    ne = ggml_ne(src)
    if out is None:
        out = ggml_empty([1, ne[1], ne[2], ne[3]], device=src.device)
    vs, vd = view_of(src), view_of(out)
    _check(lib().trc_cuda_sum_rows(ctypes.byref(vs), ctypes.byref(vd), 1 if mean else 0, _stream(stream)),
           "trc_cuda_sum_rows")
    return out


def _params6(params) -> ctypes.Array:
    vals = [float(x) for x in params]
    if len(vals) != 6:
        raise TrcCudaError("optimizer steps take six op parameters")
    return (ctypes.c_float * 6)(*vals)


def _flat(t: torch.Tensor, what: str) -> int:
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise TrcCudaError(f"{what} must be a contiguous float32 CUDA tensor")
    return t.data_ptr()


def opt_step_adamw_(param: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor, params6,
                    stream=None) -> None:
    """In-place AdamW step (the optimizer's OP_OPT_STEP_ADAMW node); params6 = {step_sz, bc2_sqrt,
    decay, beta1, beta2, eps}."""
    n = param.numel()
    if not (grad.numel() == m.numel() == v.numel() == n):
        raise TrcCudaError("opt_step_adamw: tensors differ in size")
    _check(lib().trc_cuda_opt_step_adamw(_flat(param, "param"), _flat(grad, "grad"), _flat(m, "m"), _flat(v, "v"), n,
                                         _params6(params6), _stream(stream)), "trc_cuda_opt_step_adamw")


def opt_step_sgd_(param: torch.Tensor, grad: torch.Tensor, momentum: torch.Tensor, params6, stream=None) -> None:
    """In-place SGD step (OP_OPT_STEP_SGD); params6 = {lr, momentum, dampening, weight_decay,
    nesterov, is_first}."""
    n = param.numel()
    if not (grad.numel() == momentum.numel() == n):
        raise TrcCudaError("opt_step_sgd: tensors differ in size")
    _check(lib().trc_cuda_opt_step_sgd(_flat(param, "param"), _flat(grad, "grad"), _flat(momentum, "momentum"), n,
                                       _params6(params6), _stream(stream)), "trc_cuda_opt_step_sgd")


def sum_sqr_acc_(acc: torch.Tensor, a: torch.Tensor, stream=None) -> None:
    """acc[0] += sum of a^2 (double accumulation), the clip graph's OP_SUM_SQR_ACC."""
    n = a.numel()
    ws_bytes = int(lib().trc_cuda_sum_sqr_workspace_bytes(n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device)
    _check(lib().trc_cuda_sum_sqr_acc(_flat(acc, "acc"), _flat(a, "a"), n, ws.data_ptr(), ws_bytes, _stream(stream)),
           "trc_cuda_sum_sqr_acc")


def clip_scale_(a: torch.Tensor, norm: torch.Tensor, max_norm: float, eps: float = 1e-6, stream=None) -> None:
    """a *= min(1, max_norm / (sqrt(norm[0]) + eps)), the clip graph's OP_CLIP_SCALE_INPLACE."""
    _check(lib().trc_cuda_clip_scale_inplace(_flat(a, "a"), a.numel(), _flat(norm, "norm"), max_norm, eps,
                                             _stream(stream)), "trc_cuda_clip_scale_inplace")
