"""vox_b200 — B200 (sm_100a) backend for Vox's memory-bound operator path, Python host side.

This module binds the C ABI of ``libvox_cuda.so`` (declared in ``include/vox_cuda.h``) with ctypes and exposes
one function per Vox operator, under the names of Vox's CPU operator API (``src/kernels.hpp``, ``src/nn.hpp``)
but batched and on device tensors. torch is used only to hold device memory and to name the current CUDA stream;
every operator runs a kernel of ``libvox_cuda.so``. There is no CPU fallback: if the library is missing or the
tensors are not on a CUDA device the call raises.

Errors of the library come back as :class:`VoxCudaError` carrying Vox's status code (``include/vox.h:48-55``)
and the library's per-thread message.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

__all__ = [
    "VoxCudaError", "lib", "lib_path", "version",
    "rmsnorm", "layernorm", "layer_norm", "adaln", "gated_add", "bias_add",
    "softmax_rows", "silu_mul", "swiglu_fused", "gelu", "add", "mul", "snake", "load_snake",
    "dequant_q8", "dequant_q4", "row_reduce", "global_sum_partials", "global_sum_finish", "global_sum",
    "fill_philox", "rope_inv_freq", "rope_table", "qkv_rope", "add_rmsnorm", "gemv_q8", "gemv_q4", "gemm_q8", "gemm_q4", "gemm_bf16", "Comm", "global_sum_comm", "Tmod", "F5Dit", "F32", "BF16", "F16",
]

F32, BF16, F16 = 0, 1, 2
GELU_ERF, GELU_TANH = 0, 1
SNAKE_HIFT, SNAKE_BETA, SNAKE_KOKORO = 0, 1, 2
REDUCE_SUM, REDUCE_MAX, REDUCE_L2 = 0, 1, 2
GLOBAL_SUM_SLOTS = 840
STATUS_NAMES = {-1: "VOX_ERR_IO", -2: "VOX_ERR_FORMAT", -3: "VOX_ERR_DEVICE", -4: "VOX_ERR_OOM", -6: "VOX_ERR_ARG",
                -8: "VOX_ERR_UNSUPPORTED"}

_DIR = Path(__file__).resolve().parent
lib_path = Path(os.environ.get("VOX_CUDA_LIB", _DIR / "libvox_cuda.so"))


class VoxCudaError(RuntimeError):
    """A vox_cuda call returned a negative status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def _load() -> ctypes.CDLL:
    if not lib_path.exists():
        raise ImportError(f"{lib_path} is missing: build it with `python -m vox_b200.build` (nvcc, sm_100a)")
    L = ctypes.CDLL(str(lib_path))
    c_i64, c_int, c_f, c_p, c_u64, c_u32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32
    sigs = {
        "vox_cuda_version": ([], ctypes.c_char_p),
        "vox_cuda_last_error": ([], ctypes.c_char_p),
        "vox_cuda_device_count": ([c_p], c_int),
        "vox_cuda_device_cc": ([c_p], c_int),
        "vox_cuda_device_error": ([c_p], c_int),
        "vox_cuda_test_row_stall": ([c_i64, c_u64], c_int),
        "vox_cuda_fill_philox": ([c_p, c_i64, c_int, c_f, c_f, c_u64, c_u32, c_i64, c_int, c_p], c_int),
        "vox_cuda_rmsnorm": ([c_p, c_p, c_p, c_i64, c_i64, c_f, c_int, c_p], c_int),
        "vox_cuda_layernorm": ([c_p, c_p, c_p, c_p, c_i64, c_i64, c_f, c_int, c_int, c_p], c_int),
        "vox_cuda_adaln": ([c_p, c_p, c_p, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_f, c_int, c_p], c_int),
        "vox_cuda_gated_add": ([c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_bias_add": ([c_p, c_p, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_softmax_rows": ([c_p, c_p, c_i64, c_i64, c_f, c_i64, c_i64, c_p], c_int),
        "vox_cuda_silu_mul": ([c_p, c_p, c_p, c_i64, c_int, c_p], c_int),
        "vox_cuda_swiglu_fused": ([c_p, c_p, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_gelu": ([c_p, c_p, c_i64, c_int, c_int, c_p], c_int),
        "vox_cuda_add": ([c_p, c_p, c_p, c_i64, c_int, c_p], c_int),
        "vox_cuda_mul": ([c_p, c_p, c_p, c_i64, c_int, c_p], c_int),
        "vox_cuda_snake": ([c_p, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_snake_beta_params": ([c_p, c_p, c_p, c_p, c_i64, c_p], c_int),
        "vox_cuda_dequant_q8": ([c_p, c_p, c_int, c_p, c_int, c_i64, c_i64, c_p], c_int),
        "vox_cuda_dequant_q4": ([c_p, c_p, c_int, c_p, c_int, c_i64, c_i64, c_p], c_int),
        "vox_cuda_row_reduce": ([c_p, c_p, c_i64, c_i64, c_int, c_int, c_p], c_int),
        "vox_cuda_global_sum_partials": ([c_p, c_i64, c_i64, c_i64, c_i64, c_p, c_p, c_int, c_p], c_int),
        "vox_cuda_global_sum_finish": ([c_p, c_p, c_p], c_int),
        "vox_cuda_rope_table": ([c_p, c_i64, c_i64, c_i64, c_p, c_p], c_int),
        "vox_cuda_qkv_rope": ([c_p, c_p, c_p, c_p, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f, c_p], c_int),
        "vox_cuda_add_rmsnorm": ([c_p, c_p, c_p, c_p, c_p, c_i64, c_i64, c_f, c_int, c_p], c_int),
        "vox_cuda_comm_unique_id": ([c_p], c_int),
        "vox_cuda_comm_init_rank": ([c_p, c_int, c_int, c_int, c_p], c_int),
        "vox_cuda_comm_wait": ([c_p, c_p, c_int], c_int),
        "vox_cuda_comm_destroy": ([c_p], None),
        "vox_cuda_global_sum": ([c_p, c_i64, c_i64, c_i64, c_i64, c_p, c_p, c_p, c_int, c_p, c_p], c_int),
        "vox_cuda_gemm_q8": ([c_p, c_p, c_int, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_gemm_q4": ([c_p, c_p, c_int, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_gemm_bf16": ([c_p, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_int, c_p], c_int),
        "vox_cuda_gemv_q8": ([c_p, c_p, c_int, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_gemv_q4": ([c_p, c_p, c_int, c_p, c_p, c_p, c_i64, c_i64, c_i64, c_int, c_p], c_int),
        "vox_cuda_tmod_open": ([ctypes.c_char_p, c_p], c_int),
        "vox_cuda_tmod_close": ([c_p], None),
        "vox_cuda_tmod_count": ([c_p, c_p], c_int),
        "vox_cuda_tmod_name": ([c_p, c_i64, c_p], c_int),
        "vox_cuda_tmod_info": ([c_p, ctypes.c_char_p, c_p, c_p, c_p, c_p], c_int),
        "vox_cuda_tmod_data": ([c_p, ctypes.c_char_p, c_p], c_int),
        "vox_cuda_tmod_upload": ([c_p, c_p, c_i64, c_p, c_p], c_int),
        "vox_cuda_tmod_upload_dequant": ([c_p, ctypes.c_char_p, c_p, c_int, c_p], c_int),
        "vox_cuda_f5_create": ([c_p, c_p, c_p], c_int),
        "vox_cuda_f5_buffers": ([c_p, c_p, c_p, c_p], c_int),
        "vox_cuda_f5_inputs": ([c_p, c_p, c_p], c_int),
        "vox_cuda_f5_run": ([c_p, c_p], c_int),
        "vox_cuda_f5_destroy": ([c_p], None),
    }
    for name, (args, res) in sigs.items():
        f = getattr(L, name)
        f.argtypes, f.restype = args, res
    return L


class _Lib:
    """The loaded library, opened on first use: ``vox_b200.build`` stays importable before the library exists (a
    fresh checkout), while every operator call needs it and raises ImportError when it is missing or stale."""

    _L: ctypes.CDLL | None = None

    def __getattr__(self, name: str):
        if _Lib._L is None:
            _Lib._L = _load()
        return getattr(_Lib._L, name)


lib = _Lib()


def version() -> str:
    return lib.vox_cuda_version().decode()


def device_error() -> int:
    """Device-side error bits raised since the last call (bit 0: a bounded wait gave up), then cleared."""
    flags = ctypes.c_uint(0)
    _check(lib.vox_cuda_device_error(ctypes.byref(flags)))
    return flags.value


def _check(rc: int) -> None:
    if rc != 0:
        raise VoxCudaError(rc, lib.vox_cuda_last_error().decode(errors="replace"))


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dev(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise VoxCudaError(-6, f"{name} must be a CUDA tensor (vox_b200 has no CPU path)")
    if not t.is_contiguous():
        raise VoxCudaError(-6, f"{name} must be contiguous")
    return t


def _act(t: torch.Tensor, name: str) -> int:
    _dev(t, name)
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise VoxCudaError(-6, f"{name} must be float32 or bfloat16, got {t.dtype}")


def _f32(t: torch.Tensor | None, name: str) -> int | None:
    if t is None:
        return None
    _dev(t, name)
    if t.dtype != torch.float32:
        raise VoxCudaError(-6, f"{name} must be float32 (Vox keeps this vector as const float *)")
    return t.data_ptr()


def _same(a: torch.Tensor, b: torch.Tensor, na: str, nb: str) -> None:
    if a.dtype != b.dtype or a.device != b.device:
        raise VoxCudaError(-6, f"{na} and {nb} must share dtype and device")


def _ptr(t):
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------ normalisation

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows of x [..., n] -> w * x / sqrt(mean(x^2) + eps). vox::rmsnorm (kernels.hpp:103) batched; out may be x."""
    dt = _act(x, "x")
    n = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _same(x, out, "x", "out")
    _check(lib.vox_cuda_rmsnorm(x.data_ptr(), _f32(w, "w"), out.data_ptr(), x.numel() // n, n, eps, dt, _stream(x)))
    return out


def layernorm(x, w=None, b=None, eps: float = 1e-5, modulate: bool = False, out=None) -> torch.Tensor:
    """vox::layernorm (kernels.hpp:104) / vox::nn::layer_norm (nn.hpp:83) over the last dim; modulate = (1+w)·n + b."""
    dt = _act(x, "x")
    n = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _same(x, out, "x", "out")
    _check(lib.vox_cuda_layernorm(x.data_ptr(), _f32(w, "w"), _f32(b, "b"), out.data_ptr(), x.numel() // n, n, eps,
                                  int(modulate), dt, _stream(x)))
    return out


def layer_norm(x: torch.Tensor, w, b, eps: float, modulate: bool = False) -> torch.Tensor:
    """In place, as vox::nn::layer_norm(x, T, C, w, b, eps, modulate) (nn.cpp:248-265)."""
    return layernorm(x, w, b, eps, modulate, out=x)


def adaln(x, shift, scale, eps: float = 1e-6, gate=None, residual=None, out=None) -> torch.Tensor:
    """Fused F5 adaLN over x [B][T][D]: residual + gate * (LN(x)·(1+scale) + shift), or the modulate part alone.

    shift/scale/gate: [B][D] in x's dtype. f5.cpp:617-632 (modulate) composed with f5.cpp:670-676 (gated_add).
    """
    dt = _act(x, "x")
    B, T, D = x.shape
    for t, nm in ((shift, "shift"), (scale, "scale"), (gate, "gate"), (residual, "residual")):
        if t is not None:
            _same(x, _dev(t, nm), "x", nm)
    out = torch.empty_like(x) if out is None else out
    _check(lib.vox_cuda_adaln(x.data_ptr(), shift.data_ptr(), scale.data_ptr(), _ptr(gate), _ptr(residual), out.data_ptr(),
                              B, T, D, eps, dt, _stream(x)))
    return out


def gated_add(h: torch.Tensor, gate: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """h [B][T][D] += gate [B][D] * src, in place (F5 gated_add, f5.cpp:670-676)."""
    dt = _act(h, "h")
    _same(h, _dev(src, "src"), "h", "src")
    _same(h, _dev(gate, "gate"), "h", "gate")
    B, T, D = h.shape
    _check(lib.vox_cuda_gated_add(h.data_ptr(), gate.data_ptr(), src.data_ptr(), B, T, D, dt, _stream(h)))
    return h


def bias_add(y: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """y [..., D] += b [D] in place (bias loop of vox::nn::linear, nn.cpp:148-155)."""
    dt = _act(y, "y")
    D = y.shape[-1]
    _check(lib.vox_cuda_bias_add(y.data_ptr(), _f32(b, "b"), y.numel() // D, D, dt, _stream(y)))
    return y


# ------------------------------------------------------------------ softmax

def softmax_rows(x: torch.Tensor, scale: float = 1.0, q_len: int = 0, pos0: int = 0, out=None) -> torch.Tensor:
    """Scaled row softmax of f32 rows [..., n]; q_len > 0 applies Vox's causal truncation (kernels.cpp:812-819)."""
    if _act(x, "x") != F32:
        raise VoxCudaError(-6, "softmax_rows works on float32 scores")
    n = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _same(x, out, "x", "out")
    _check(lib.vox_cuda_softmax_rows(x.data_ptr(), out.data_ptr(), x.numel() // n, n, scale, q_len, pos0, _stream(x)))
    return out


# ------------------------------------------------------------------ activations

def silu_mul(g: torch.Tensor, u: torch.Tensor, out=None) -> torch.Tensor:
    """silu(g) * u (the SwiGLU loop of kernels.cpp:836); out may be g."""
    dt = _act(g, "g")
    _same(g, _dev(u, "u"), "g", "u")
    out = torch.empty_like(g) if out is None else out
    _check(lib.vox_cuda_silu_mul(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), dt, _stream(g)))
    return out


def swiglu_fused(gu: torch.Tensor, out=None) -> torch.Tensor:
    """gu [m][2I] -> silu(gu[:, :I]) * gu[:, I:] (swiglu.comp)."""
    dt = _act(gu, "gu")
    m, I2 = gu.shape
    out = torch.empty((m, I2 // 2), dtype=gu.dtype, device=gu.device) if out is None else out
    _check(lib.vox_cuda_swiglu_fused(gu.data_ptr(), out.data_ptr(), m, I2 // 2, dt, _stream(gu)))
    return out


def gelu(x: torch.Tensor, kind: int = GELU_ERF, out=None) -> torch.Tensor:
    """GELU, erf form (vox::gelu_erf, nn::gelu_inplace) or tanh form (F5 gelu_tanh); out may be x."""
    dt = _act(x, "x")
    out = torch.empty_like(x) if out is None else out
    _same(x, out, "x", "out")
    _check(lib.vox_cuda_gelu(x.data_ptr(), out.data_ptr(), x.numel(), kind, dt, _stream(x)))
    return out


def add(a: torch.Tensor, b: torch.Tensor, out=None) -> torch.Tensor:
    dt = _act(a, "a")
    _same(a, _dev(b, "b"), "a", "b")
    out = torch.empty_like(a) if out is None else out
    _check(lib.vox_cuda_add(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), dt, _stream(a)))
    return out


def mul(a: torch.Tensor, b: torch.Tensor, out=None) -> torch.Tensor:
    dt = _act(a, "a")
    _same(a, _dev(b, "b"), "a", "b")
    out = torch.empty_like(a) if out is None else out
    _check(lib.vox_cuda_mul(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), dt, _stream(a)))
    return out


def snake(x: torch.Tensor, alpha: torch.Tensor, kind: int = SNAKE_HIFT, beta=None, channel_major: bool = True,
          out=None) -> torch.Tensor:
    """Snake over f32 x: channel_major -> x [..., C, T] (inner = T); else Vox's time-major [T][C] (inner = 1)."""
    if _act(x, "x") != F32:
        raise VoxCudaError(-6, "snake works on float32 activations")
    C = alpha.numel()
    inner = x.shape[-1] if channel_major else 1
    out = torch.empty_like(x) if out is None else out
    _check(lib.vox_cuda_snake(x.data_ptr(), _f32(alpha, "alpha"), _f32(beta, "beta"), out.data_ptr(), x.numel(), C, inner,
                              kind, _stream(x)))
    return out


def load_snake(alpha: torch.Tensor, beta: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The Snake struct of load_snake (qwen3.cpp:76-84): a = exp(alpha), inv_b = 1/(exp(beta) + 1e-9)."""
    a = torch.empty_like(alpha)
    ib = torch.empty_like(beta)
    _check(lib.vox_cuda_snake_beta_params(_f32(alpha, "alpha"), _f32(beta, "beta"), a.data_ptr(), ib.data_ptr(), alpha.numel(),
                                          _stream(alpha)))
    return a, ib


# ------------------------------------------------------------------ dequantisation

def _scale_dt(scale: torch.Tensor) -> int:
    _dev(scale, "scale")
    if scale.dtype == torch.float32:
        return F32
    if scale.dtype == torch.float16:
        return F16
    raise VoxCudaError(-6, "scale must be float32 (Vox's layout) or float16")


def dequant_q8(q: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16, out=None) -> torch.Tensor:
    """int8 q [rows][cols] * scale [rows][cols/32] -> out (vox::mat_row Q8, kernels.cpp:446-452)."""
    _dev(q, "q")
    rows, cols = q.shape
    out = torch.empty((rows, cols), dtype=out_dtype, device=q.device) if out is None else out
    _check(lib.vox_cuda_dequant_q8(q.data_ptr(), scale.data_ptr(), _scale_dt(scale), out.data_ptr(), _act(out, "out"), rows, cols,
                                   _stream(q)))
    return out


def dequant_q4(q: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16, out=None) -> torch.Tensor:
    """packed uint8 q [rows][cols/2] -> out [rows][cols] (vox::mat_row Q4, kernels.cpp:453-463)."""
    _dev(q, "q")
    rows, half = q.shape
    cols = half * 2
    out = torch.empty((rows, cols), dtype=out_dtype, device=q.device) if out is None else out
    _check(lib.vox_cuda_dequant_q4(q.data_ptr(), scale.data_ptr(), _scale_dt(scale), out.data_ptr(), _act(out, "out"), rows, cols,
                                   _stream(q)))
    return out


# ------------------------------------------------------------------ reductions

def row_reduce(x: torch.Tensor, op: int = REDUCE_SUM, out=None) -> torch.Tensor:
    """Per-row sum / max / L2 norm of x [..., n] -> f32 [...]."""
    dt = _act(x, "x")
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device) if out is None else out
    _check(lib.vox_cuda_row_reduce(x.data_ptr(), out.data_ptr(), rows, n, op, dt, _stream(x)))
    return out


def global_sum_partials(x: torch.Tensor, row0: int, total_rows: int, slots=None, scratch=None) -> torch.Tensor:
    """Slot partials (f64 [840]) of this shard's rows [row0, row0 + rows) of a [total_rows][n] tensor."""
    dt = _act(x, "x")
    n = x.shape[-1]
    rows = x.numel() // n
    slots = torch.empty(GLOBAL_SUM_SLOTS, dtype=torch.float64, device=x.device) if slots is None else slots
    scratch = torch.empty(max(rows, 1), dtype=torch.float32, device=x.device) if scratch is None else scratch
    _check(lib.vox_cuda_global_sum_partials(x.data_ptr(), rows, n, row0, total_rows, scratch.data_ptr(), slots.data_ptr(), dt,
                                            _stream(x)))
    return slots


def global_sum_finish(slots: torch.Tensor, out=None) -> torch.Tensor:
    out = torch.empty(1, dtype=torch.float64, device=slots.device) if out is None else out
    _check(lib.vox_cuda_global_sum_finish(slots.data_ptr(), out.data_ptr(), _stream(slots)))
    return out


def global_sum(x: torch.Tensor, row0: int = 0, total_rows: int | None = None, group=None) -> torch.Tensor:
    """Deterministic sum of a row-sharded tensor: slot partials, one all-reduce of 840 f64 (NCCL), fixed-order fold.

    With torch.distributed initialised, every rank passes its shard and the global row offset; the result (f64 [1])
    is bitwise identical for any world size that divides the rows into whole slots.
    """
    total_rows = x.numel() // x.shape[-1] if total_rows is None else total_rows
    slots = global_sum_partials(x, row0, total_rows)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(slots, op=dist.ReduceOp.SUM, group=group)
    return global_sum_finish(slots)


class Comm:
    """A communicator of the library over the shards' GPUs (vox_cuda_comm_*: NCCL, non-blocking, with deadlines), one
    rank per process. Rank 0 draws ``Comm.unique_id()`` and hands the bytes to every rank (any channel)."""

    ID_BYTES = 128

    def __init__(self, uid: bytes, nranks: int, rank: int, timeout_ms: int = 30000):
        buf = ctypes.create_string_buffer(bytes(uid), self.ID_BYTES)
        h = ctypes.c_void_p()
        _check(lib.vox_cuda_comm_init_rank(buf, nranks, rank, timeout_ms, ctypes.byref(h)))
        self.h, self.nranks, self.rank = h, nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(Comm.ID_BYTES)
        _check(lib.vox_cuda_comm_unique_id(buf))
        return buf.raw

    def wait(self, timeout_ms: int = 0, stream=None) -> None:
        """Waits until the current (or given) stream's work is done; raises (and aborts the communicator) past the
        deadline or on an NCCL error."""
        st = torch.cuda.current_stream().cuda_stream if stream is None else stream
        _check(lib.vox_cuda_comm_wait(self.h, st, timeout_ms))

    def close(self) -> None:
        if self.h:
            lib.vox_cuda_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def global_sum_comm(x: torch.Tensor, row0: int, total_rows: int, comm: Comm | None, slots=None, scratch=None, out=None) -> torch.Tensor:
    """The deterministic global sum of a row-sharded tensor in one library call (partials, all-reduce over ``comm``,
    fold): f64 [1], bitwise identical on every rank and for any number of ranks."""
    dt = _act(x, "x")
    n = x.shape[-1]
    rows = x.numel() // n
    slots = torch.empty(GLOBAL_SUM_SLOTS, dtype=torch.float64, device=x.device) if slots is None else slots
    scratch = torch.empty(max(rows, 1), dtype=torch.float32, device=x.device) if scratch is None else scratch
    out = torch.empty(1, dtype=torch.float64, device=x.device) if out is None else out
    _check(lib.vox_cuda_global_sum(x.data_ptr(), rows, n, row0, total_rows, scratch.data_ptr(), slots.data_ptr(), out.data_ptr(), dt,
                                   comm.h if comm is not None else None, _stream(x)))
    return out


# ------------------------------------------------------------------ synthetic data

def fill_philox(out: torch.Tensor, dist: int, a: float, b: float, seed: int = 0, stream_id: int = 0, counter0: int = 0) -> torch.Tensor:
    """Fill a device tensor with Vox's Philox4x32-10 draws (0 uniform, 1 normal, 2 int8 codes, 3 bytes)."""
    _dev(out, "out")
    dt = BF16 if out.dtype == torch.bfloat16 else F32
    _check(lib.vox_cuda_fill_philox(out.data_ptr(), out.numel(), dist, a, b, seed, stream_id, counter0, dt, _stream(out)))
    return out


# ------------------------------------------------------------------ transformer elementwise chain

def rope_inv_freq(hd: int, theta: float, device="cuda") -> torch.Tensor:
    """vox::rope_inv_freq (kernels.cpp:734-738): float(1 / theta^(2i/hd)) computed in double, as a device tensor.
    A model-load-time constant (host arithmetic, then one copy), not a per-step operator."""
    v = [float(1.0 / (float(theta) ** (2.0 * i / hd))) for i in range(hd // 2)]
    return torch.tensor(v, dtype=torch.float32).to(device)


def rope_table(inv_freq: torch.Tensor, pos0: int, m: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """cos/sin table [m][half][2] of positions pos0 .. pos0+m-1 (the table of gpu_vulkan.cpp:855-860), on the device."""
    half = inv_freq.numel()
    out = torch.empty((m, half, 2), dtype=torch.float32, device=inv_freq.device) if out is None else out
    _f32(out, "out")
    _check(lib.vox_cuda_rope_table(_f32(inv_freq, "inv_freq"), half, pos0, m, out.data_ptr(), _stream(inv_freq)))
    return out


def qkv_rope(qkv: torch.Tensor, cs: torch.Tensor, heads: int, kv_heads: int, hd: int, k_cache: torch.Tensor,
             v_cache: torch.Tensor, pos0: int, q_norm_w=None, k_norm_w=None, ring: int = 0, eps: float = 1e-6,
             q: torch.Tensor | None = None) -> torch.Tensor:
    """Split the fused projection qkv [m][(heads + 2 kv_heads) hd], head-RMSNorm and RoPE q and k, write q and the
    tokens' K/V cache rows (pos0 + i, or (pos0 + i) % ring). Returns q [m][heads hd]. qkvsplit.comp + qkrope.comp,
    CPU form kernels.cpp:797-806."""
    _f32(qkv, "qkv")
    m = qkv.numel() // ((heads + 2 * kv_heads) * hd)
    q = torch.empty((m, heads * hd), dtype=torch.float32, device=qkv.device) if q is None else q
    _check(lib.vox_cuda_qkv_rope(qkv.data_ptr(), _f32(q_norm_w, "q_norm_w"), _f32(k_norm_w, "k_norm_w"), _f32(cs, "cs"),
                                 _f32(q, "q"), _f32(k_cache, "k_cache"), _f32(v_cache, "v_cache"), m, heads, kv_heads, hd,
                                 pos0, ring, eps, _stream(qkv)))
    return q


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float, layer_scale=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """h += delta (* layer_scale) in place, then returns rmsnorm(h) * w (kernels.cpp:822-825 then 833)."""
    dt = _act(h, "h")
    _same(h, delta, "h", "delta")
    n = h.shape[-1]
    out = torch.empty_like(h) if out is None else out
    _same(h, out, "h", "out")
    _check(lib.vox_cuda_add_rmsnorm(h.data_ptr(), delta.data_ptr(), _f32(layer_scale, "layer_scale"), _f32(w, "w"),
                                    out.data_ptr(), h.numel() // n, n, eps, dt, _stream(h)))
    return out


# ------------------------------------------------------------------ GEMM on the tensor cores

GEMM_NONE, GEMM_GELU_ERF, GEMM_GELU_TANH = 0, 1, 2


def gemm_bf16(x: torch.Tensor, w: torch.Tensor, bias=None, act: int = GEMM_NONE, out_dtype=torch.float32, out=None) -> torch.Tensor:
    """y [m][n] = act(x [m][k] . w [n][k]^T + bias [n]) on the tensor cores: bf16 x and w, f32 accumulation, y f32 or
    bf16 (the GEMM of gpu_f5.cpp:287-322 / gemmb.comp with its bias and GELU flags)."""
    for t, nm in ((x, "x"), (w, "w")):
        _dev(t, nm)
        if t.dtype != torch.bfloat16:
            raise VoxCudaError(-6, f"{nm} must be bfloat16")
    k = x.shape[-1]
    if w.dim() != 2 or w.shape[1] != k:
        raise VoxCudaError(-6, "w must be [n][k] with x's k")
    m, n = x.numel() // k, w.shape[0]
    od = F32 if out_dtype == torch.float32 else BF16
    out = torch.empty(*x.shape[:-1], n, dtype=out_dtype, device=x.device) if out is None else out
    _check(lib.vox_cuda_gemm_bf16(x.data_ptr(), w.data_ptr(), _f32(bias, "bias"), out.data_ptr(), m, n, k, act, od, _stream(x)))
    return out


# ------------------------------------------------------------------ quantized GEMV (decode)

def _gemv(fn, q4, w, scale, x, bias, out, accumulate):
    _dev(w, "w")
    if w.dtype != (torch.uint8 if q4 else torch.int8):
        raise VoxCudaError(-6, f"w must be {'uint8 (packed Q4)' if q4 else 'int8'}")
    sdt = _scale_dt(scale)
    xf = _f32(x, "x")
    rows, cols = w.shape[0], x.shape[-1]
    m = x.numel() // cols
    if out is None:
        out = torch.zeros((m, rows), dtype=torch.float32, device=x.device) if accumulate else \
            torch.empty((m, rows), dtype=torch.float32, device=x.device)
    _check(fn(w.data_ptr(), scale.data_ptr(), sdt, _f32(bias, "bias"), xf, _f32(out, "out"), rows, cols, m, int(accumulate),
              _stream(x)))
    return out


def gemv_q8(w: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, bias=None, out=None, accumulate: bool = False) -> torch.Tensor:
    """y [m][rows] = W x (+ bias), W = int8 codes [rows][cols] x scale [rows][cols/32] (f32 or f16); the GPU matvec
    of matmul.comp (float activations). accumulate adds into out."""
    return _gemv(lib.vox_cuda_gemv_q8, False, w, scale, x, bias, out, accumulate)


def gemv_q4(w: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, bias=None, out=None, accumulate: bool = False) -> torch.Tensor:
    """As gemv_q8 with Q4 weights: uint8 [rows][cols/2], 16 bytes per 32-block (byte j = code j | code j+16 << 4)."""
    return _gemv(lib.vox_cuda_gemv_q4, True, w, scale, x, bias, out, accumulate)


def gemm_q8(w: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, bias=None, out=None, accumulate: bool = False) -> torch.Tensor:
    """The prefill form of gemv_q8 (many activation rows) on the tensor cores in f16: y [m][rows] = W x (+ bias)."""
    return _gemv(lib.vox_cuda_gemm_q8, False, w, scale, x, bias, out, accumulate)


def gemm_q4(w: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, bias=None, out=None, accumulate: bool = False) -> torch.Tensor:
    """The prefill form of gemv_q4 on the tensor cores in f16."""
    return _gemv(lib.vox_cuda_gemm_q4, True, w, scale, x, bias, out, accumulate)


# ------------------------------------------------------------------ .tmod weight files -> device

TMOD_DTYPES = ["F32", "F16", "BF16", "I32", "I16", "I8", "U8"]  # Vox's DType order (src/common.hpp:22)
_TORCH_OF = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "I32": torch.int32, "I16": torch.int16,
             "I8": torch.int8, "U8": torch.uint8}


class Tmod:
    """A mapped .tmod file (vox::TmodFile, src/formats.hpp:65-84): blob names, descriptions, host views, and uploads
    to the device through pinned staging (vox_cuda_tmod_upload); Q8/Q4 matrices can be dequantised on arrival."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib.vox_cuda_tmod_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib.vox_cuda_tmod_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        n = ctypes.c_int64()
        _check(lib.vox_cuda_tmod_count(self._h, ctypes.byref(n)))
        out = []
        for i in range(n.value):
            p = ctypes.c_char_p()
            _check(lib.vox_cuda_tmod_name(self._h, i, ctypes.byref(p)))
            out.append(p.value.decode())
        return out

    def info(self, name: str) -> tuple[str, tuple, int]:
        """(dtype name, shape, nbytes) of a blob."""
        dt, nd, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        shape = (ctypes.c_int64 * 8)()
        _check(lib.vox_cuda_tmod_info(self._h, name.encode(), ctypes.byref(dt), shape, ctypes.byref(nd), ctypes.byref(nb)))
        return TMOD_DTYPES[dt.value], tuple(shape[i] for i in range(nd.value)), nb.value

    def host_bytes(self, name: str) -> bytes:
        """A copy of the blob's bytes from the mapping (no device work)."""
        p = ctypes.c_void_p()
        _check(lib.vox_cuda_tmod_data(self._h, name.encode(), ctypes.byref(p)))
        return ctypes.string_at(p.value, self.info(name)[2])

    def upload(self, names, outs=None, device="cuda"):
        """Copies blobs to the device (one call, pinned staging, the current stream); returns the tensors."""
        names = [names] if isinstance(names, str) else list(names)
        if outs is None:
            outs = []
            for n in names:
                dt, shape, nb = self.info(n)
                outs.append(torch.empty(shape, dtype=_TORCH_OF[dt], device=device))
        for t in outs:
            _dev(t, "out")
        cn = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        dp = (ctypes.c_void_p * len(outs))(*[t.data_ptr() for t in outs])
        st = _stream(outs[0]) if outs else 0
        _check(lib.vox_cuda_tmod_upload(self._h, ctypes.cast(cn, ctypes.c_void_p), len(names), ctypes.cast(dp, ctypes.c_void_p), st))
        return outs

    def upload_dequant(self, name: str, out_dtype=torch.bfloat16, device="cuda") -> torch.Tensor:
        """The Q8/Q4 matrix `name` (+ "<name>.scale") dequantised on the device to [rows][cols] (mat_row, bit-exact)."""
        dt, shape, _ = self.info(name)
        rows, cols = shape[0], (shape[1] if len(shape) > 1 else 1) * (2 if dt == "U8" else 1)
        out = torch.empty((rows, cols), dtype=out_dtype, device=device)
        _check(lib.vox_cuda_tmod_upload_dequant(self._h, name.encode(), out.data_ptr(), _act(out, "out"), _stream(out)))
        return out


# ------------------------------------------------------------------ F5 DiT step (one CUDA graph)

class _F5Block(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ("ada", "q", "k", "v", "o", "ff1", "ff2", "ada_b", "q_b", "k_b", "v_b", "o_b", "ff1_b",
                                              "ff2_b")]


class _F5Desc(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int32) for k in ("dim", "heads", "dim_head", "ff_mult", "depth", "pe_attn_head", "out_dim", "batch",
                                              "frames", "math")] + \
               [("blocks", ctypes.POINTER(_F5Block)), ("norm_out", ctypes.c_void_p), ("proj_out", ctypes.c_void_p),
                ("norm_out_b", ctypes.c_void_p), ("proj_out_b", ctypes.c_void_p), ("in_dim", ctypes.c_int32)] + \
               [(k, ctypes.c_void_p) for k in ("in_proj", "in_proj_b", "pos1_w", "pos1_b", "pos2_w", "pos2_b")]


class _DevView:
    """A device buffer of the library exposed to torch without a copy (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3, "strides": None}


class F5Dit:
    """The transformer of one F5-TTS DiT step (Vox's gpu_f5_step, gpu_f5.cpp:273-332; CPU F5Model::dit,
    f5.cpp:608-724) from the residual stream h after the input embedding to the output projection, captured once as a
    CUDA graph (vox_cuda_f5_create) and replayed by run(). `blocks` is a list of dicts of f32 CUDA tensors
    {ada [6D][D], q/k/v [H*HD][D], o [D][H*HD], ff1 [F][D], ff2 [D][F]} in Vox's [out][in] layout, each with an
    optional bias "<name>_b" [out] (absent: zero); norm_out [2D][D] gives (scale, shift), proj_out [out_dim][D], with
    optional biases norm_out_b, proj_out_b. `embed` (optional) adds the input embedding: a dict {in_proj [D][in_dim],
    in_proj_b, pos1_w, pos2_w [D][D/16][31], pos1_b, pos2_b}; the step then starts from x [rows][out_dim] and cond
    [rows][in_dim - out_dim] (condition mel, then text embedding). `math`: "f32" (CUDA-core GEMMs), "tf32" or "bf16"
    (tensor cores, f32 accumulation). h, ts, out (and x, cond) are the plan's own buffers (torch views, valid until
    close())."""

    MATH = {"f32": 0, "tf32": 1, "bf16": 2}
    KEYS = ("ada", "q", "k", "v", "o", "ff1", "ff2")

    def __init__(self, blocks, norm_out, proj_out, *, heads: int, dim_head: int, batch: int, frames: int,
                 pe_attn_head: int = 0, math: str = "tf32", norm_out_b=None, proj_out_b=None, embed: dict | None = None):
        if math not in self.MATH:
            raise VoxCudaError(-6, f"math must be one of {sorted(self.MATH)}")
        D = int(norm_out.shape[1])
        inner, out_dim = heads * dim_head, int(proj_out.shape[0])
        ff = int(blocks[0]["ff1"].shape[0]) if blocks else 0
        if not blocks or ff % D:
            raise VoxCudaError(-6, "blocks must be non-empty and ff1 rows a multiple of dim")
        want = {"ada": (6 * D, D), "q": (inner, D), "k": (inner, D), "v": (inner, D), "o": (D, inner), "ff1": (ff, D), "ff2": (D, ff)}
        def check(t, nm, shp):
            if t is None:
                return None
            if _dev(t, nm).dtype != torch.float32 or tuple(t.shape) != shp:
                raise VoxCudaError(-6, f"{nm} must be f32 {shp}")
            return t.data_ptr()

        for i, b in enumerate(blocks):
            for k, shp in want.items():
                check(b[k], f"blocks[{i}].{k}", shp)
                check(b.get(k + "_b"), f"blocks[{i}].{k}_b", shp[:1])
        check(norm_out, "norm_out", (2 * D, D))
        check(proj_out, "proj_out", (out_dim, D))
        nb, pb = check(norm_out_b, "norm_out_b", (2 * D,)), check(proj_out_b, "proj_out_b", (out_dim,))
        emb = [0] + [None] * 6
        if embed is not None:
            in_dim = int(embed["in_proj"].shape[1])
            cw = (D, D // 16, 31)
            emb = [in_dim, check(embed["in_proj"], "in_proj", (D, in_dim)), check(embed.get("in_proj_b"), "in_proj_b", (D,)),
                   check(embed["pos1_w"], "pos1_w", cw), check(embed.get("pos1_b"), "pos1_b", (D,)),
                   check(embed["pos2_w"], "pos2_w", cw), check(embed.get("pos2_b"), "pos2_b", (D,))]
        self._keep = (blocks, norm_out, proj_out, norm_out_b, proj_out_b, embed)  # read by every run
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        arr = (_F5Block * len(blocks))(*[_F5Block(*([b[k].data_ptr() for k in self.KEYS] + [ptr(b.get(k + "_b")) for k in self.KEYS]))
                                         for b in blocks])
        desc = _F5Desc(D, heads, dim_head, ff // D, len(blocks), pe_attn_head, out_dim, batch, frames, self.MATH[math], arr,
                       norm_out.data_ptr(), proj_out.data_ptr(), nb, pb, *emb)
        h = ctypes.c_void_p()
        _check(lib.vox_cuda_f5_create(ctypes.byref(desc), _stream(norm_out), ctypes.byref(h)))
        self._h = h
        ph, pts, po = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib.vox_cuda_f5_buffers(self._h, ctypes.byref(ph), ctypes.byref(pts), ctypes.byref(po)))
        R = batch * frames
        self.h = torch.as_tensor(_DevView(ph.value, (R, D)), device=norm_out.device)
        self.ts = torch.as_tensor(_DevView(pts.value, (D,)), device=norm_out.device)
        self.out = torch.as_tensor(_DevView(po.value, (R, out_dim)), device=norm_out.device)
        self.x = self.cond = None
        if embed is not None:
            px, pc = ctypes.c_void_p(), ctypes.c_void_p()
            _check(lib.vox_cuda_f5_inputs(self._h, ctypes.byref(px), ctypes.byref(pc)))
            self.x = torch.as_tensor(_DevView(px.value, (R, out_dim)), device=norm_out.device)
            self.cond = torch.as_tensor(_DevView(pc.value, (R, emb[0] - out_dim)), device=norm_out.device)

    def run(self) -> None:
        """Replays the step on the current stream: reads ts and h (or x and cond), updates h, writes out."""
        _check(lib.vox_cuda_f5_run(self._h, _stream(self.h)))

    def step(self, h: torch.Tensor | None, ts: torch.Tensor, x: torch.Tensor | None = None,
             cond: torch.Tensor | None = None) -> torch.Tensor:
        """Copies the inputs in (h [batch*frames][dim], or x and cond with the embedding), runs the step, returns a
        copy of out."""
        if self.x is None:
            self.h.copy_(h.reshape(self.h.shape))
        else:
            self.x.copy_(x.reshape(self.x.shape))
            self.cond.copy_(cond.reshape(self.cond.shape))
        self.ts.copy_(ts.reshape(self.ts.shape))
        self.run()
        return self.out.clone()

    def close(self) -> None:
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.h.device)
            lib.vox_cuda_f5_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
