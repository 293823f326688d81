"""TEST INFRASTRUCTURE — numpy front end of the parity oracles. Not product code.

``port()`` loads the plain-C restatement of Vox's CPU arithmetic (``oracle/vox_oracle.c`` ->
``oracle/_build/libvox_oracle.so``, compiled on demand with gcc). ``ref()`` loads dariumi/Vox's own CPU operators
compiled from the reference sources (``oracle/_ref/libvox_ref.so``, built by ``make -C oracle ref`` where the
reference sources exist) or returns None when that library is absent.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use this module.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "_build" / "libvox_oracle.so"
REF_SO = HERE / "_ref" / "libvox_ref.so"

_f = ctypes.c_float
_d = ctypes.c_double
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_p = ctypes.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def build_port() -> Path:
    src = HERE / "vox_oracle.c"
    if not PORT_SO.exists() or PORT_SO.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    return PORT_SO


def reference_dir() -> Path | None:
    """The reference's source root: $VOX_REFERENCE_DIR, else a directory named ``reference`` beside this repository's
    root; None where neither holds the reference sources (on a GPU box only the prebuilt oracle/_ref travels)."""
    import os

    for cand in (os.environ.get("VOX_REFERENCE_DIR"), str(HERE.parent.parent / "reference")):
        if cand and (Path(cand) / "src" / "kernels.cpp").exists():
            return Path(cand)
    return None


def build_ref(ref_root: str | Path | None = None) -> Path | None:
    root = Path(ref_root) if ref_root is not None else reference_dir()
    if root is None or not (root / "src" / "kernels.cpp").exists():
        return REF_SO if REF_SO.exists() else None
    shim = HERE / "ref_shim.cpp"
    if not REF_SO.exists() or REF_SO.stat().st_mtime < shim.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={root}"], check=True)
    return REF_SO


class Port:
    """The C restatement (vox_oracle.c), numpy in / numpy out."""

    def __init__(self):
        self.L = L = ctypes.CDLL(str(build_port()))
        L.vo_uniform.restype = _f
        L.vo_uniform.argtypes = [_u64, _u64, _u32, _u32]
        L.vo_f16_to_f32.restype = _f
        L.vo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.vo_f32_to_bf16.restype = ctypes.c_uint16
        L.vo_f32_to_bf16.argtypes = [_f]
        L.vo_fast_sin.restype = _f
        L.vo_fast_sin.argtypes = [_f]
        L.vo_global_sum_finish.restype = _d
        L.vo_global_sum_finish.argtypes = [_p]
        L.vo_fill.argtypes = [_p, _i64, _int, _f, _f, _u64, _u32, _i64]
        L.vo_fill_i8.argtypes = [_p, _i64, _int, _int, _u64, _u32, _i64]
        L.vo_fill_u8.argtypes = [_p, _i64, _u64, _u32, _i64]
        L.vo_f5_noise.argtypes = [_u64, _u32, _i64, _p]
        L.vo_rmsnorm_rows.argtypes = [_p, _p, _i64, _i64, _f, _p]
        L.vo_layernorm_rows.argtypes = [_p, _p, _p, _i64, _i64, _f, _int, _p]
        L.vo_modulate.argtypes = [_p, _p, _p, _i64, _i64, _d, _p]
        L.vo_gated_add.argtypes = [_p, _p, _p, _i64, _i64]
        L.vo_adaln.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _d, _p]
        L.vo_bias_add.argtypes = [_p, _p, _i64, _i64]
        L.vo_softmax_rows.argtypes = [_p, _p, _i64, _i64, _f, _i64, _i64]
        L.vo_silu_mul.argtypes = [_p, _p, _p, _i64]
        L.vo_swiglu_fused.argtypes = [_p, _p, _i64, _i64]
        L.vo_gelu_erf.argtypes = [_p, _p, _i64]
        L.vo_gelu_tanh.argtypes = [_p, _p, _i64]
        L.vo_add.argtypes = [_p, _p, _p, _i64]
        L.vo_mul.argtypes = [_p, _p, _p, _i64]
        L.vo_snake.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _int]
        L.vo_load_snake.argtypes = [_p, _p, _p, _p, _i64]
        L.vo_dequant_q8.argtypes = [_p, _p, _i64, _i64, _p]
        L.vo_dequant_q4.argtypes = [_p, _p, _i64, _i64, _p]
        L.vo_row_reduce_ordered.argtypes = [_p, _p, _i64, _i64, _int, _int]
        L.vo_row_reduce_f64.argtypes = [_p, _p, _i64, _i64, _int]
        L.vo_global_sum_slots.argtypes = [_p, _i64, _i64, _i64, _p]
        L.vo_philox_block.argtypes = [_p, _p, _p]
        L.vo_f32_to_bf16_n.argtypes = [_p, _p, _i64]
        L.vo_f16_to_f32_n.argtypes = [_p, _p, _i64]
        L.vo_rope_inv_freq.argtypes = [_i64, _d, _p]
        L.vo_rope_table.argtypes = [_p, _i64, _i64, _i64, _p]
        L.vo_qkv_rope.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f]
        L.vo_add_rmsnorm.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _f]
        L.vo_gemv.argtypes = [_int, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int]

    # -- generator
    def philox_block(self, ctr, key):
        c, k, o = _c(ctr, np.uint32), _c(key, np.uint32), np.zeros(4, np.uint32)
        self.L.vo_philox_block(_ptr(c), _ptr(k), _ptr(o))
        return o

    def uniform(self, seed, frame, codebook, draw=0):
        return self.L.vo_uniform(seed, frame, codebook, draw)

    def fill(self, n, dist, a, b, seed=0, sid=0, c0=0):
        out = np.empty(n, np.float32)
        self.L.vo_fill(_ptr(out), n, dist, a, b, seed, sid, c0)
        return out

    def normal(self, shape, mean=0.0, std=1.0, seed=0, sid=0, c0=0):
        return self.fill(int(np.prod(shape)), 1, mean, std, seed, sid, c0).reshape(shape)

    def uniform_arr(self, shape, lo, hi, seed=0, sid=0, c0=0):
        return self.fill(int(np.prod(shape)), 0, lo, hi, seed, sid, c0).reshape(shape)

    def fill_into(self, out, dist, a=0.0, b=1.0, seed=0, sid=0, c0=0, threads=None):
        """Fill a preallocated contiguous array with the numbers of ``fill`` / ``fill_i8`` / ``fill_u8`` (dist 0 / 1:
        f32, 2: int8 codes in [a, b], 3: bytes), split over host threads (each element depends only on its counter)."""
        import concurrent.futures as cf
        import os

        flat = out.reshape(-1)
        n = flat.size
        threads = threads or os.cpu_count() or 1
        step = max(1 << 16, -(-n // (4 * threads)))
        step += step & 1  # even chunk starts (Box-Muller pairs)

        def one(lo):
            hi = min(n, lo + step)
            ptr = flat[lo:hi].ctypes.data_as(_p)
            if dist in (0, 1):
                self.L.vo_fill(ptr, hi - lo, dist, a, b, seed, sid, c0 + lo)
            elif dist == 2:
                self.L.vo_fill_i8(ptr, hi - lo, int(a), int(b), seed, sid, c0 + lo)
            else:
                self.L.vo_fill_u8(ptr, hi - lo, seed, sid, c0 + lo)

        with cf.ThreadPoolExecutor(threads) as ex:
            list(ex.map(one, range(0, n, step)))
        return out

    def bf16_round_into(self, x, out, threads=None):
        """bf16 bits of f32 x into the preallocated uint16 ``out`` (build.py:94-97), split over host threads."""
        import concurrent.futures as cf
        import os

        xf, of = x.reshape(-1), out.reshape(-1)
        n = xf.size
        threads = threads or os.cpu_count() or 1
        step = max(1 << 16, -(-n // (4 * threads)))
        with cf.ThreadPoolExecutor(threads) as ex:
            list(ex.map(lambda lo: self.L.vo_f32_to_bf16_n(xf[lo:lo + step].ctypes.data_as(_p), of[lo:lo + step].ctypes.data_as(_p),
                                                           min(step, n - lo)), range(0, n, step)))
        return out

    def fill_i8(self, shape, a, b, seed=0, sid=0, c0=0):
        out = np.empty(int(np.prod(shape)), np.int8)
        self.L.vo_fill_i8(_ptr(out), out.size, a, b, seed, sid, c0)
        return out.reshape(shape)

    def fill_u8(self, shape, seed=0, sid=0, c0=0):
        out = np.empty(int(np.prod(shape)), np.uint8)
        self.L.vo_fill_u8(_ptr(out), out.size, seed, sid, c0)
        return out.reshape(shape)

    def f5_noise(self, seed, chunk, n):
        out = np.empty(n, np.float32)
        self.L.vo_f5_noise(seed, chunk, n, _ptr(out))
        return out

    # -- conversions
    def bf16_round(self, x):
        """f32 -> bf16 bits (python/vox/build.py:94-97)."""
        x = _c(x, np.float32)
        out = np.empty(x.shape, np.uint16)
        self.L.vo_f32_to_bf16_n(_ptr(x), _ptr(out), x.size)
        return out

    def f16_to_f32(self, h):
        h = _c(h, np.uint16)
        out = np.empty(h.shape, np.float32)
        self.L.vo_f16_to_f32_n(_ptr(h), _ptr(out), h.size)
        return out

    # -- normalisation
    def rmsnorm(self, x, w, eps):
        x, w = _c(x, np.float32), _c(w, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vo_rmsnorm_rows(_ptr(x), _ptr(w), x.size // n, n, eps, _ptr(out))
        return out

    def layernorm(self, x, w, b, eps, modulate=False):
        x = _c(x, np.float32)
        w = None if w is None else _c(w, np.float32)
        b = None if b is None else _c(b, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vo_layernorm_rows(_ptr(x), _ptr(w), _ptr(b), x.size // n, n, eps, int(modulate), _ptr(out))
        return out

    def adaln(self, x, shift, scale, gate=None, res=None, eps=1e-6):
        x, shift, scale = _c(x, np.float32), _c(shift, np.float32), _c(scale, np.float32)
        gate = None if gate is None else _c(gate, np.float32)
        res = None if res is None else _c(res, np.float32)
        B, T, D = x.shape
        out = np.empty_like(x)
        self.L.vo_adaln(_ptr(x), _ptr(shift), _ptr(scale), _ptr(gate), _ptr(res), B, T, D, float(eps), _ptr(out))
        return out

    def gated_add(self, h, gate, src):
        """h [B][T][D] += gate[b] * src, on a copy."""
        h = _c(h, np.float32).copy()
        gate, src = _c(gate, np.float32), _c(src, np.float32)
        B, T, D = h.shape
        for bb in range(B):
            hb = np.ascontiguousarray(h[bb])
            self.L.vo_gated_add(_ptr(hb), _ptr(np.ascontiguousarray(gate[bb])), _ptr(np.ascontiguousarray(src[bb])), T, D)
            h[bb] = hb
        return h

    def bias_add(self, y, b):
        y = _c(y, np.float32).copy()
        b = _c(b, np.float32)
        D = y.shape[-1]
        self.L.vo_bias_add(_ptr(y), _ptr(b), y.size // D, D)
        return y

    # -- softmax
    def softmax_rows(self, x, scale=1.0, q_len=0, pos0=0):
        x = _c(x, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vo_softmax_rows(_ptr(x), _ptr(out), x.size // n, n, scale, q_len, pos0)
        return out

    # -- activations
    def silu_mul(self, g, u):
        g, u = _c(g, np.float32), _c(u, np.float32)
        out = np.empty_like(g)
        self.L.vo_silu_mul(_ptr(g), _ptr(u), _ptr(out), g.size)
        return out

    def swiglu_fused(self, gu):
        gu = _c(gu, np.float32)
        m, I2 = gu.shape
        out = np.empty((m, I2 // 2), np.float32)
        self.L.vo_swiglu_fused(_ptr(gu), _ptr(out), m, I2 // 2)
        return out

    def gelu(self, x, kind=0):
        x = _c(x, np.float32)
        out = np.empty_like(x)
        (self.L.vo_gelu_erf if kind == 0 else self.L.vo_gelu_tanh)(_ptr(x), _ptr(out), x.size)
        return out

    def add(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.empty_like(a)
        self.L.vo_add(_ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def mul(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.empty_like(a)
        self.L.vo_mul(_ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def snake(self, x, alpha, kind=0, beta=None, inner=1):
        x, alpha = _c(x, np.float32), _c(alpha, np.float32)
        beta = None if beta is None else _c(beta, np.float32)
        out = np.empty_like(x)
        self.L.vo_snake(_ptr(x), _ptr(alpha), _ptr(beta), _ptr(out), x.size, alpha.size, inner, kind)
        return out

    def load_snake(self, alpha, beta):
        alpha, beta = _c(alpha, np.float32), _c(beta, np.float32)
        a, ib = np.empty_like(alpha), np.empty_like(beta)
        self.L.vo_load_snake(_ptr(alpha), _ptr(beta), _ptr(a), _ptr(ib), alpha.size)
        return a, ib

    def fast_sin(self, x):
        return self.L.vo_fast_sin(float(x))

    # -- dequantisation (f32 scales; convert f16 scales with f16_to_f32 first)
    def dequant_q8(self, q, scale):
        q, scale = _c(q, np.int8), _c(scale, np.float32)
        rows, cols = q.shape
        out = np.empty((rows, cols), np.float32)
        self.L.vo_dequant_q8(_ptr(q), _ptr(scale), rows, cols, _ptr(out))
        return out

    def dequant_q4(self, q, scale):
        q, scale = _c(q, np.uint8), _c(scale, np.float32)
        rows, half = q.shape
        out = np.empty((rows, half * 2), np.float32)
        self.L.vo_dequant_q4(_ptr(q), _ptr(scale), rows, half * 2, _ptr(out))
        return out

    # -- reductions
    def row_reduce(self, x, op=0, W=4):
        """The CUDA kernel's fixed order (W = 4 for f32 inputs, 8 for bf16 inputs given here as f32)."""
        x = _c(x, np.float32)
        n = x.shape[-1]
        out = np.empty(x.size // n, np.float32)
        self.L.vo_row_reduce_ordered(_ptr(x), _ptr(out), x.size // n, n, op, W)
        return out.reshape(x.shape[:-1])

    def row_reduce_f64(self, x, op=0):
        x = _c(x, np.float32)
        n = x.shape[-1]
        out = np.empty(x.size // n, np.float64)
        self.L.vo_row_reduce_f64(_ptr(x), _ptr(out), x.size // n, n, op)
        return out.reshape(x.shape[:-1])

    def global_sum_slots(self, rowsum, row0, total_rows):
        rowsum = _c(rowsum, np.float32)
        slots = np.empty(840, np.float64)
        self.L.vo_global_sum_slots(_ptr(rowsum), row0, rowsum.size, total_rows, _ptr(slots))
        return slots

    def global_sum_finish(self, slots):
        slots = _c(slots, np.float64)
        return self.L.vo_global_sum_finish(_ptr(slots))

    # -- transformer elementwise chain
    def rope_inv_freq(self, hd, theta):
        out = np.empty(hd // 2, np.float32)
        self.L.vo_rope_inv_freq(hd, theta, _ptr(out))
        return out

    def rope_table(self, inv_freq, pos0, m):
        inv_freq = _c(inv_freq, np.float32)
        cs = np.empty((m, inv_freq.size, 2), np.float32)
        self.L.vo_rope_table(_ptr(inv_freq), inv_freq.size, pos0, m, _ptr(cs))
        return cs

    def qkv_rope(self, qkv, qn, kn, cs, heads, kv_heads, hd, pos0=0, kc=None, vc=None, ring=0, eps=1e-6):
        """Returns (q, k_cache, v_cache); the caches are copied (default: pos0 + m zero rows, or ring rows)."""
        qkv = _c(qkv, np.float32)
        m = qkv.shape[0]
        kd = kv_heads * hd
        rows = ring if ring > 0 else pos0 + m
        kc = np.zeros((rows, kd), np.float32) if kc is None else _c(kc, np.float32).copy()
        vc = np.zeros((rows, kd), np.float32) if vc is None else _c(vc, np.float32).copy()
        q = np.empty((m, heads * hd), np.float32)
        qn = None if qn is None else _c(qn, np.float32)
        kn = None if kn is None else _c(kn, np.float32)
        cs = _c(cs, np.float32)
        self.L.vo_qkv_rope(_ptr(qkv), _ptr(qn), _ptr(kn), _ptr(cs), _ptr(q), _ptr(kc), _ptr(vc), m, heads, kv_heads, hd, pos0,
                           ring, eps)
        return q, kc, vc

    def gemv(self, q, scale, x, bias=None, y=None, q4=False):
        """y [m][rows] = W x (+ bias) (y given: accumulate into a copy of it); returns (y, bound) where bound is
        sum_k |W[r][k] x[i][k]|. q: int8 [rows][cols] or packed uint8 [rows][cols/2]; scale f32 [rows][cols/32]."""
        q = np.ascontiguousarray(q)
        scale, x = _c(scale, np.float32), _c(x, np.float32)
        rows, cols = q.shape[0], x.shape[-1]
        m = x.size // cols
        acc = y is not None
        y = np.zeros((m, rows), np.float32) if y is None else _c(y, np.float32).copy()
        bound = np.empty((m, rows), np.float64)
        bias = None if bias is None else _c(bias, np.float32)
        self.L.vo_gemv(int(q4), _ptr(q), _ptr(scale), _ptr(bias), _ptr(x), _ptr(y), _ptr(bound), rows, cols, m, int(acc))
        return y, bound

    def add_rmsnorm(self, h, d, ls, w, eps=1e-6):
        """Returns (h + d * ls, rmsnorm of it)."""
        h = _c(h, np.float32).copy()
        d, w = _c(d, np.float32), _c(w, np.float32)
        ls = None if ls is None else _c(ls, np.float32)
        n = h.shape[-1]
        xn = np.empty_like(h)
        self.L.vo_add_rmsnorm(_ptr(h), _ptr(d), _ptr(ls), _ptr(w), _ptr(xn), h.size // n, n, eps)
        return h, xn


class Ref:
    """dariumi/Vox's own CPU operators (oracle/_ref/libvox_ref.so), numpy in / numpy out."""

    def __init__(self, path: Path):
        self.L = L = ctypes.CDLL(str(path))
        L.vr_uniform.restype = _f
        L.vr_uniform.argtypes = [_u64, _u64, _u32, _u32]
        L.vr_f16_to_f32.restype = _f
        L.vr_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.vr_fast_sin.restype = _f
        L.vr_fast_sin.argtypes = [_f]
        L.vr_num_threads.restype = _int
        L.vr_set_threads.argtypes = [_int]
        L.vr_philox_block.argtypes = [_p, _p, _p]
        L.vr_f5_noise.argtypes = [_u64, _u32, _i64, _p]
        L.vr_rmsnorm_rows.argtypes = [_p, _p, _i64, _i64, _f, _p, _int]
        L.vr_layernorm_rows.argtypes = [_p, _p, _p, _i64, _i64, _f, _p]
        L.vr_nn_layer_norm.argtypes = [_p, _int, _int, _p, _p, _f, _int]
        L.vr_adaln.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p]
        L.vr_bias_add.argtypes = [_p, _p, _i64, _i64]
        L.vr_softmax_rows.argtypes = [_p, _p, _i64, _i64, _f, _i64, _i64, _int]
        L.vr_silu_mul.argtypes = [_p, _p, _p, _i64]
        L.vr_gelu_erf.argtypes = [_p, _p, _i64]
        L.vr_gelu_inplace.argtypes = [_p, _i64]
        L.vr_gelu_tanh.argtypes = [_p, _p, _i64]
        L.vr_add.argtypes = [_p, _p, _p, _i64]
        L.vr_mul.argtypes = [_p, _p, _p, _i64]
        L.vr_snake.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _int]
        L.vr_mat_rows.argtypes = [_int, _p, _p, _i64, _i64, _p]
        L.vr_quantize_q8.argtypes = [_p, _i64, _i64, _p, _p]
        L.vr_quantize_q4.argtypes = [_p, _i64, _i64, _p, _p]
        L.vr_row_reduce.argtypes = [_p, _p, _i64, _i64, _int]
        L.vr_rope_inv_freq.argtypes = [_i64, _d, _p]
        L.vr_qk_norm_rope.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f]
        L.vr_add_rmsnorm.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _f]
        L.vr_matmul.argtypes = [_int, _p, _p, _p, _i64, _i64, _p, _i64, _p]
        L.vr_tmod_write.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _i64, _p, _p, _p, _p, _p, _p, _u32]
        L.vr_tmod_write.restype = _int
        L.vr_tmod_read.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _p, _u64]
        L.vr_tmod_read.restype = _i64
        for nm, args in (("vr_gelu_f32", [_p, _p, _i64]), ("vr_gelu_bf16", [_p, _p, _i64]), ("vr_add_bf16", [_p, _p, _p, _i64]),
                         ("vr_mul_bf16", [_p, _p, _p, _i64]), ("vr_row_reduce_bf16", [_p, _p, _i64, _i64, _int]),
                         ("vr_mat_rows_bf16", [_int, _p, _p, _i64, _i64, _p]),
                         ("vr_adaln_bf16", [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p])):
            if hasattr(L, nm):
                getattr(L, nm).argtypes = args
        if hasattr(L, "vr_global_sum"):
            L.vr_global_sum.argtypes = [_p, _i64, _i64, _p, _p]
            L.vr_global_sum.restype = _d
        if hasattr(L, "vr_f5_dit"):
            L.vr_f5_dit.argtypes = [ctypes.c_char_p, _int, _int, _p, _p, _p, _f, _p, _p, ctypes.c_char_p, _int]
            L.vr_f5_dit.restype = _int

    def set_threads(self, n: int) -> int:
        self.L.vr_set_threads(n)
        return self.L.vr_num_threads()

    def philox_block(self, ctr, key):
        c, k, o = _c(ctr, np.uint32), _c(key, np.uint32), np.zeros(4, np.uint32)
        self.L.vr_philox_block(_ptr(c), _ptr(k), _ptr(o))
        return o

    def uniform(self, seed, frame, codebook, draw=0):
        return self.L.vr_uniform(seed, frame, codebook, draw)

    def f5_noise(self, seed, chunk, n):
        out = np.empty(n, np.float32)
        self.L.vr_f5_noise(seed, chunk, n, _ptr(out))
        return out

    def f16_to_f32(self, h):
        return np.array([self.L.vr_f16_to_f32(int(v)) for v in np.asarray(h, np.uint16).ravel()], np.float32).reshape(np.shape(h))

    def rmsnorm(self, x, w, eps, par=1):
        x, w = _c(x, np.float32), _c(w, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vr_rmsnorm_rows(_ptr(x), _ptr(w), x.size // n, n, eps, _ptr(out), par)
        return out

    def layernorm(self, x, w, b, eps):
        x, w = _c(x, np.float32), None if w is None else _c(w, np.float32)
        b = None if b is None else _c(b, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vr_layernorm_rows(_ptr(x), _ptr(w), _ptr(b), x.size // n, n, eps, _ptr(out))
        return out

    def nn_layer_norm(self, x, w, b, eps, modulate=False):
        x = _c(x, np.float32).copy()
        w = None if w is None else _c(w, np.float32)
        b = None if b is None else _c(b, np.float32)
        T, C = x.shape
        self.L.vr_nn_layer_norm(_ptr(x), T, C, _ptr(w), _ptr(b), eps, int(modulate))
        return x

    def adaln(self, x, shift, scale, gate=None, res=None):
        x, shift, scale = _c(x, np.float32), _c(shift, np.float32), _c(scale, np.float32)
        gate = None if gate is None else _c(gate, np.float32)
        res = None if res is None else _c(res, np.float32)
        B, T, D = x.shape
        out = np.empty_like(x)
        self.L.vr_adaln(_ptr(x), _ptr(shift), _ptr(scale), _ptr(gate), _ptr(res), B, T, D, _ptr(out))
        return out

    def bias_add(self, y, b):
        y = _c(y, np.float32).copy()
        b = _c(b, np.float32)
        D = y.shape[-1]
        self.L.vr_bias_add(_ptr(y), _ptr(b), y.size // D, D)
        return y

    def softmax_rows(self, x, scale=1.0, q_len=0, pos0=0, fast=False):
        x = _c(x, np.float32)
        n = x.shape[-1]
        out = np.empty_like(x)
        self.L.vr_softmax_rows(_ptr(x), _ptr(out), x.size // n, n, scale, q_len, pos0, int(fast))
        return out

    def silu_mul(self, g, u):
        g, u = _c(g, np.float32), _c(u, np.float32)
        out = np.empty_like(g)
        self.L.vr_silu_mul(_ptr(g), _ptr(u), _ptr(out), g.size)
        return out

    def gelu_erf(self, x):
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self.L.vr_gelu_erf(_ptr(x), _ptr(out), x.size)
        return out

    def gelu_inplace(self, x):
        x = _c(x, np.float32).copy()
        self.L.vr_gelu_inplace(_ptr(x), x.size)
        return x

    def gelu_tanh(self, x):
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self.L.vr_gelu_tanh(_ptr(x), _ptr(out), x.size)
        return out

    def add(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.empty_like(a)
        self.L.vr_add(_ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def mul(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.empty_like(a)
        self.L.vr_mul(_ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def snake(self, x, alpha, kind=0, beta=None, inner=1):
        x, alpha = _c(x, np.float32), _c(alpha, np.float32)
        beta = None if beta is None else _c(beta, np.float32)
        out = np.empty_like(x)
        self.L.vr_snake(_ptr(x), _ptr(alpha), _ptr(beta), _ptr(out), x.size, alpha.size, inner, kind)
        return out

    def fast_sin(self, x):
        return self.L.vr_fast_sin(float(x))

    def mat_rows(self, q, scale, q4=False):
        scale = _c(scale, np.float32)
        if q4:
            q = _c(q, np.uint8)
            rows, cols = q.shape[0], q.shape[1] * 2
        else:
            q = _c(q, np.int8)
            rows, cols = q.shape
        out = np.empty((rows, cols), np.float32)
        self.L.vr_mat_rows(4 if q4 else 3, _ptr(q), _ptr(scale), rows, cols, _ptr(out))
        return out

    def quantize_q8(self, w):
        w = _c(w, np.float32)
        rows, cols = w.shape
        q, s = np.empty((rows, cols), np.int8), np.empty((rows, cols // 32), np.float32)
        self.L.vr_quantize_q8(_ptr(w), rows, cols, _ptr(q), _ptr(s))
        return q, s

    def quantize_q4(self, w):
        w = _c(w, np.float32)
        rows, cols = w.shape
        q, s = np.empty((rows, cols // 2), np.uint8), np.empty((rows, cols // 32), np.float32)
        self.L.vr_quantize_q4(_ptr(w), rows, cols, _ptr(q), _ptr(s))
        return q, s

    def row_reduce(self, x, op=0):
        x = _c(x, np.float32)
        n = x.shape[-1]
        out = np.empty(x.size // n, np.float32)
        self.L.vr_row_reduce(_ptr(x), _ptr(out), x.size // n, n, op)
        return out

    def rope_inv_freq(self, hd, theta):
        out = np.empty(hd // 2, np.float32)
        self.L.vr_rope_inv_freq(hd, theta, _ptr(out))
        return out

    def qk_norm_rope(self, q, k, qn, kn, inv_freq, heads, kv_heads, hd, pos0=0, eps=1e-6):
        """transformer_forward's q/k step on split projections; returns new (q, k)."""
        q, k = _c(q, np.float32).copy(), _c(k, np.float32).copy()
        qn = None if qn is None else _c(qn, np.float32)
        kn = None if kn is None else _c(kn, np.float32)
        inv_freq = _c(inv_freq, np.float32)
        self.L.vr_qk_norm_rope(_ptr(q), _ptr(k), _ptr(qn), _ptr(kn), _ptr(inv_freq), q.shape[0], heads, kv_heads, hd, pos0, eps)
        return q, k

    def matmul(self, wtype, data, scale, x, rows, cols, bias=None):
        """vox::matmul on a CPU Mat (wtype 0 F32, 3 Q8, 4 Q4): y [m][rows]."""
        data = np.ascontiguousarray(data)
        scale = None if scale is None else _c(scale, np.float32)
        bias = None if bias is None else _c(bias, np.float32)
        x = _c(x, np.float32)
        m = x.size // cols
        y = np.empty((m, rows), np.float32)
        self.L.vr_matmul(wtype, _ptr(data), _ptr(scale), _ptr(bias), rows, cols, _ptr(x), m, _ptr(y))
        return y

    def tmod_write(self, path, manifest_json: str, blobs: dict, flags: int = 0) -> None:
        """vox::tmod_write; blobs: name -> (dtype code, shape, bytes)."""
        names = list(blobs)
        cnames = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        dts = np.array([blobs[n][0] for n in names], np.int32)
        shapes = np.zeros((len(names), 8), np.int64)
        nd = np.array([len(blobs[n][1]) for n in names], np.int32)
        for i, n in enumerate(names):
            shapes[i, :len(blobs[n][1])] = blobs[n][1]
        bufs = [ctypes.create_string_buffer(bytes(blobs[n][2]), max(1, len(blobs[n][2]))) for n in names]
        ptrs = (ctypes.c_void_p * len(names))(*[ctypes.addressof(b) for b in bufs])
        nb = np.array([len(blobs[n][2]) for n in names], np.uint64)
        rc = self.L.vr_tmod_write(str(path).encode(), manifest_json.encode(), len(names), ctypes.cast(cnames, _p), _ptr(dts),
                                  _ptr(shapes), _ptr(nd), ctypes.cast(ptrs, _p), _ptr(nb), flags)
        if rc != 0:
            raise RuntimeError("vox::tmod_write failed")

    def f5_dit(self, path, x, cond, temb, t: float, dim: int):
        """F5Model(path) on the CPU: (time_embed(t) [dim], dit_forward(B, N, x, cond, temb, t) [B][N][mel_dim])."""
        x, cond, temb = _c(x, np.float32), _c(cond, np.float32), _c(temb, np.float32)
        B, N, M = x.shape
        ts, out = np.empty(dim, np.float32), np.empty((B, N, M), np.float32)
        err = ctypes.create_string_buffer(512)
        if self.L.vr_f5_dit(str(path).encode(), B, N, _ptr(x), _ptr(cond), _ptr(temb), float(t), _ptr(ts), _ptr(out), err, 512) != 0:
            raise RuntimeError("F5Model: " + err.value.decode(errors="replace"))
        return ts, out

    def tmod_read(self, path, name: str) -> bytes | None:
        """vox::TmodFile(path).get(name) bytes, or None (missing blob or bad file)."""
        n = self.L.vr_tmod_read(str(path).encode(), name.encode(), None, 0)
        if n < 0:
            return None
        buf = ctypes.create_string_buffer(max(1, n))
        self.L.vr_tmod_read(str(path).encode(), name.encode(), buf, n)
        return buf.raw[:n]

    def add_rmsnorm(self, h, d, ls, w, eps=1e-6):
        h = _c(h, np.float32).copy()
        d, w = _c(d, np.float32), _c(w, np.float32)
        ls = None if ls is None else _c(ls, np.float32)
        n = h.shape[-1]
        xn = np.empty_like(h)
        self.L.vr_add_rmsnorm(_ptr(h), _ptr(d), _ptr(ls), _ptr(w), _ptr(xn), h.size // n, n, eps)
        return h, xn


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def ref() -> Ref | None:
    global _ref
    if _ref is None:
        p = build_ref()
        if p is None or not p.exists():
            return None
        _ref = Ref(p)
    return _ref


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_f32(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (RNE, build.py:94-97) and return it as f32 values."""
    return bf16_bits_to_f32(port().bf16_round(x))
