"""Python front of libnebw (include/nebw.h) through ctypes.

This module is plumbing for tests, the benchmark and Python callers: the
product is the C ABI and the CUDA kernels behind it.  There is no CPU path
here: if libnebw.so is missing or no sm_100 GPU is present, the calls fail
by name.

Device buffers may be torch CUDA tensors (their data_ptr is passed) or raw
integer device addresses.
"""

from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent.parent          # npu-embeddings-xdna1_b200/
REPO_DIR = PKG_DIR.parent
LIB_PATH = Path(os.environ["NEBW_LIB"]) if os.environ.get("NEBW_LIB") else PKG_DIR / "libnebw.so"
HEADER_PATH = REPO_DIR / "include" / "nebw.h"

F32, BF16 = 0, 1
ACT_NONE, ACT_GELU8, ACT_GELU_ERF = 0, 1, 2
GATE_SILU, GATE_GELU_ERF = 0, 1
POOL_MEAN, POOL_CLS = 0, 1


class NebwError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nebw error {code}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "num_layers", "hidden", "num_heads", "head_dim", "intermediate", "vocab_size",
        "max_seq_len", "type_vocab_size", "pooling", "l2_normalize", "activation")] + [
        ("layer_norm_eps", C.c_float)] + [(n, C.c_int32) for n in (
        "gated_ffn", "gated_act", "rope", "reserved0")] + [("rope_theta", C.c_double)]


class VitConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "num_layers", "hidden", "num_heads", "head_dim", "intermediate", "image_size",
        "patch_size", "num_channels")] + [("layer_norm_eps", C.c_float)]


_lib = None


def header_functions() -> list[str]:
    """Names of every function include/nebw.h declares."""
    text = HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nebw_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    """Load libnebw.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(
            f"{LIB_PATH} is not built; run `python __graft_entry__.py build` (or build()) first")
    L = C.CDLL(str(LIB_PATH))
    vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int32
    sig = {
        "nebw_last_error": ([], C.c_char_p),
        "nebw_abi_version": ([], C.c_int),
        "nebw_open": ([C.c_int, C.POINTER(vp)], C.c_int),
        "nebw_close": ([vp], C.c_int),
        "nebw_sync": ([vp], C.c_int),
        "nebw_alloc": ([vp, C.c_size_t, C.POINTER(vp)], C.c_int),
        "nebw_free": ([vp, vp], C.c_int),
        "nebw_copy_h2d": ([vp, vp, vp, C.c_size_t], C.c_int),
        "nebw_copy_d2h": ([vp, vp, vp, C.c_size_t], C.c_int),
        "nebw_device_info": ([vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)], C.c_int),
        "nebw_stage_weight": ([vp, vp, C.c_int, i64, i64, C.POINTER(C.c_uint64)], C.c_int),
        "nebw_release_weight": ([vp, C.c_uint64], C.c_int),
        "nebw_gemm": ([vp, C.c_uint64, vp, i64, i64, i64, vp, vp, C.c_int, vp, C.c_int, vp], C.c_int),
        "nebw_layernorm": ([vp, vp, vp, C.c_int, vp, vp, C.c_float, i64, i64, vp, vp], C.c_int),
        "nebw_attention": ([vp, vp, i64, vp, vp, i32, i32, i32, i32, vp, vp], C.c_int),
        "nebw_pack_offsets": ([vp, vp, i32, i32, vp, vp, vp], C.c_int),
        "nebw_embed_ln": ([vp, vp, vp, vp, i32, i32, vp, i32, vp, vp, vp, vp, C.c_float, i32, vp,
                           vp, vp], C.c_int),
        "nebw_pool_l2": ([vp, vp, vp, vp, i32, i32, C.c_int, C.c_int, vp, vp], C.c_int),
        "nebw_narrow_bf16": ([vp, vp, i64, vp, vp], C.c_int),
        "nebw_model_create": ([vp, C.POINTER(Config), C.POINTER(vp)], C.c_int),
        "nebw_model_set_rope_freq": ([vp, C.POINTER(C.c_double), C.c_int32], C.c_int),
        "nebw_model_set_tensor": ([vp, C.c_char_p, vp, C.c_int, i64, i64], C.c_int),
        "nebw_model_load_npue": ([vp, C.c_char_p, C.POINTER(vp)], C.c_int),
        "nebw_tma_layout_hash": ([], C.c_char_p),
        "nebw_npue_gemm_kn": ([C.c_char_p, C.c_char_p, vp, i64, i64], C.c_int),
        "nebw_model_set_gemm_nk": ([vp, C.c_char_p, vp, i64, i64], C.c_int),
        "nebw_model_destroy": ([vp], C.c_int),
        "nebw_model_get_config": ([vp, C.POINTER(Config)], C.c_int),
        "nebw_encode": ([vp, vp, vp, i32, i32, vp], C.c_int),
        "nebw_encode_device": ([vp, vp, vp, i32, i32, vp, vp], C.c_int),
        "nebw_encode_launch_count": ([vp, i32], C.c_int),
        "nebw_encode_device_static": ([vp, vp, vp, i32, i32, vp, vp], C.c_int),
        "nebw_set_attention_kernel": ([vp, C.c_int], C.c_int),
        "nebw_model_profile": ([vp, C.c_int], C.c_int),
        "nebw_model_profile_collect": ([vp, C.POINTER(C.c_int64), C.POINTER(C.c_double)], C.c_int),
        "nebw_vit_create": ([vp, C.POINTER(VitConfig), C.POINTER(vp)], C.c_int),
        "nebw_vit_set_tensor": ([vp, C.c_char_p, vp, C.c_int, i64, i64], C.c_int),
        "nebw_vit_load_npue": ([vp, C.c_char_p, C.POINTER(vp)], C.c_int),
        "nebw_vit_get_config": ([vp, C.POINTER(VitConfig)], C.c_int),
        "nebw_vit_destroy": ([vp], C.c_int),
        "nebw_vit_encode_device": ([vp, vp, i32, vp, vp], C.c_int),
        "nebw_vit_encode": ([vp, vp, i32, vp], C.c_int),
        "nebw_vit_launch_count": ([vp], C.c_int),
        "nebw_vit_profile": ([vp, C.c_int], C.c_int),
        "nebw_vit_profile_collect": ([vp, C.POINTER(C.c_int64), C.POINTER(C.c_double)], C.c_int),
        "nebw_check_bounded_wait": ([vp, i64, C.POINTER(i32)], C.c_int),
        "nebw_quantise_rows": ([vp, vp, i64, i64, vp, vp, vp, vp], C.c_int),
        "nebw_stage_weight_i8": ([vp, vp, i64, i64, C.POINTER(C.c_uint64)], C.c_int),
        "nebw_gemm_i8": ([vp, C.c_uint64, vp, vp, i64, i64, i64, vp, vp, C.c_int, vp, vp], C.c_int),
        "nebw_gemm_i8_ex": ([vp, C.c_uint64, vp, vp, i64, i64, i64, vp, vp, C.c_int, vp, C.c_int,
                             vp], C.c_int),
        "nebw_quantise_rows_bf16": ([vp, vp, i64, i64, vp, vp, vp, vp], C.c_int),
        "nebw_layernorm_quant": ([vp, vp, vp, vp, vp, C.c_float, i64, i64, vp, vp, vp, vp],
                                 C.c_int),
        "nebw_model_set_int8_operand": ([vp, C.c_char_p, vp, vp, vp, i64, i64], C.c_int),
        "nebw_model_set_datapath": ([vp, i32], C.c_int),
        "nebw_model_set_graphs": ([vp, i32], C.c_int),
        "nebw_pack_checkpoint": ([C.c_char_p, C.c_char_p, C.c_char_p, i32, i32,
                                  C.POINTER(C.c_uint64)], C.c_int),
        "nebw_comm_unique_id": ([vp], C.c_int),
        "nebw_comm_init_rank": ([vp, i32, i32, vp, C.c_double, C.POINTER(vp)], C.c_int),
        "nebw_comm_init_all": ([i32, C.POINTER(vp), C.c_double, C.POINTER(vp)], C.c_int),
        "nebw_comm_destroy": ([vp], C.c_int),
        "nebw_comm_size": ([vp, C.POINTER(i32), C.POINTER(i32)], C.c_int),
        "nebw_comm_sync": ([vp, vp], C.c_int),
        "nebw_shard_plan": ([vp, i32, i32, vp, vp], C.c_int),
        "nebw_shard_order": ([vp, i32, i32, vp], C.c_int),
        "nebw_gather_rows": ([vp, vp, vp, i32, vp, i32, vp], C.c_int),
        "nebw_encode_shard_gather": ([vp, vp, vp, vp, i32, i32, vp, vp, vp, vp], C.c_int),
        "nebw_encode_sharded": ([vp, vp, vp, vp, i32, i32, vp], C.c_int),
        "nebw_encode_multi": ([i32, C.POINTER(vp), C.POINTER(vp), vp, vp, i32, i32, vp], C.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def _check(rc: int):
    if rc != 0:
        raise NebwError(rc, lib().nebw_last_error().decode())


def _addr(x):
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream's handle


def _stream(s):
    """cudaStream_t for the C ABI.  None -> the library's own stream (NULL);
    a torch stream -> its handle, with torch's legacy default stream (handle
    0) passed as cudaStreamLegacy so that it is not read as NULL."""
    if s is None:
        return None
    h = s if isinstance(s, int) else s.cuda_stream
    return h if h != 0 else CUDA_STREAM_LEGACY


class Device:
    """One GPU (nebw_dev)."""

    def __init__(self, index: int = 0, torch_stream: bool = False):
        """torch_stream: op calls that name no stream run on torch's current
        stream (so they are ordered with the torch ops that made their
        buffers) instead of on the handle's own stream."""
        h = C.c_void_p()
        _check(lib().nebw_open(index, C.byref(h)))
        self.h = h
        self.index = index
        self.torch_stream = torch_stream

    def _s(self, stream):
        if stream is not None:
            return _stream(stream)
        if self.torch_stream:
            import torch
            return _stream(torch.cuda.current_stream())
        return None

    def close(self):
        if self.h:
            lib().nebw_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self):
        if self.torch_stream:
            import torch
            torch.cuda.current_stream().synchronize()
        _check(lib().nebw_sync(self.h))

    ATTN_MMA, ATTN_TCGEN05 = 0, 1

    def set_attention_kernel(self, kind: int):
        _check(lib().nebw_set_attention_kernel(self.h, kind))

    def check_bounded_wait(self, limit_ns: int) -> bool:
        """True if the probe's wait ran out (nebw_check_bounded_wait)."""
        e = C.c_int32()
        _check(lib().nebw_check_bounded_wait(self.h, limit_ns, C.byref(e)))
        return bool(e.value)

    def info(self):
        sm, ma, mi = C.c_int(), C.c_int(), C.c_int()
        _check(lib().nebw_device_info(self.h, C.byref(sm), C.byref(ma), C.byref(mi)))
        return {"sm_count": sm.value, "cc": (ma.value, mi.value)}

    # ---- weights and ops -------------------------------------------------
    def stage_weight(self, w_kn: np.ndarray) -> int:
        w = np.ascontiguousarray(w_kn)
        dt = F32 if w.dtype == np.float32 else BF16
        if w.dtype not in (np.float32, np.uint16):
            raise TypeError("weights are fp32, or bf16 bit patterns as uint16")
        K, N = w.shape
        hnd = C.c_uint64()
        _check(lib().nebw_stage_weight(self.h, w.ctypes.data, dt, K, N, C.byref(hnd)))
        return hnd.value

    def stage_weight_i8(self, w_kn: np.ndarray) -> int:
        """An int8 [K, N] GEMM operand (nebw_stage_weight_i8)."""
        w = np.ascontiguousarray(w_kn, np.int8)
        K, N = w.shape
        hnd = C.c_uint64()
        _check(lib().nebw_stage_weight_i8(self.h, w.ctypes.data, K, N, C.byref(hnd)))
        return hnd.value

    def gemm_i8(self, weight, A, sa, M, K, N, ws, C_out, bias=None, act=ACT_NONE, stream=None,
                c_dtype=F32):
        """C = dequant(A . W) (nebw_gemm_i8_ex): fp32 C, or bf16 RNE with c_dtype BF16."""
        _check(lib().nebw_gemm_i8_ex(self.h, weight, _addr(A), _addr(sa), M, K, N, _addr(ws),
                                     _addr(bias), act, _addr(C_out), c_dtype, self._s(stream)))

    def quantise_rows(self, x, rows, K, ias, q, scale, stream=None):
        """quantise_a_int8 per row; x fp32, or a torch bf16 tensor (widened exactly)."""
        fn = (lib().nebw_quantise_rows_bf16 if str(getattr(x, "dtype", "")) == "torch.bfloat16"
              else lib().nebw_quantise_rows)
        _check(fn(self.h, _addr(x), rows, K, _addr(ias), _addr(q), _addr(scale), self._s(stream)))

    def layernorm_quant(self, x, gamma, beta, rows, H, y=None, ias=None, q=None, scale=None,
                        eps=1e-12, stream=None):
        """add_norm_quant: x = LN(x + y) in place (y fp32 or None), then the rows
        quantised with ias into q / scale when q is given."""
        _check(lib().nebw_layernorm_quant(self.h, _addr(x), _addr(y), _addr(gamma), _addr(beta),
                                          eps, rows, H, _addr(ias), _addr(q), _addr(scale),
                                          self._s(stream)))

    def release_weight(self, handle: int):
        _check(lib().nebw_release_weight(self.h, handle))

    def gemm(self, weight, A, M, K, N, C_out, bias=None, residual=None, act=ACT_NONE,
             c_dtype=BF16, stream=None):
        _check(lib().nebw_gemm(self.h, weight, _addr(A), M, K, N, _addr(bias), _addr(residual),
                               act, _addr(C_out), c_dtype, self._s(stream)))

    def layernorm(self, x, gamma, beta, rows, H, y=None, a_bf16=None, eps=1e-12, stream=None,
                  y_dtype=None):
        """x = LN(x + y) in place; y_dtype defaults to y's own (torch bf16 -> BF16, else F32)."""
        if y_dtype is None:
            y_dtype = BF16 if str(getattr(y, "dtype", "")) == "torch.bfloat16" else F32
        _check(lib().nebw_layernorm(self.h, _addr(x), _addr(y), y_dtype, _addr(gamma),
                                    _addr(beta), eps, rows, H, _addr(a_bf16), self._s(stream)))

    def attention(self, qkv, rows, seq_off, seq_len, B, max_len, heads, head_dim, ctx, stream=None):
        _check(lib().nebw_attention(self.h, _addr(qkv), rows, _addr(seq_off), _addr(seq_len), B,
                                    max_len, heads, head_dim, _addr(ctx), self._s(stream)))

    def pack_offsets(self, len_in, B, S, len_out, seq_off, stream=None):
        _check(lib().nebw_pack_offsets(self.h, _addr(len_in), B, S, _addr(len_out),
                                       _addr(seq_off), self._s(stream)))

    def embed_ln(self, ids, seq_off, seq_len, B, S, word, vocab, pos, typ, gamma, beta, H, x,
                 a_bf16=None, eps=1e-12, stream=None):
        _check(lib().nebw_embed_ln(self.h, _addr(ids), _addr(seq_off), _addr(seq_len), B, S,
                                   _addr(word), vocab, _addr(pos), _addr(typ), _addr(gamma),
                                   _addr(beta), eps, H, _addr(x), _addr(a_bf16), self._s(stream)))

    def pool_l2(self, h, seq_off, seq_len, B, H, pooling, out, l2=True, stream=None):
        _check(lib().nebw_pool_l2(self.h, _addr(h), _addr(seq_off), _addr(seq_len), B, H,
                                  pooling, int(l2), _addr(out), self._s(stream)))

    def narrow_bf16(self, x, n, y, stream=None):
        _check(lib().nebw_narrow_bf16(self.h, _addr(x), n, _addr(y), self._s(stream)))


class Model:
    """A staged BERT encoder on one Device (nebw_model)."""

    def __init__(self, dev: Device, handle):
        self.dev = dev
        self.h = handle
        cfg = Config()
        _check(lib().nebw_model_get_config(self.h, C.byref(cfg)))
        self.cfg = cfg

    @classmethod
    def from_weights(cls, dev: Device, w, max_seq_len: int = 512, activation: int = ACT_GELU8):
        """Stage a nebw.synth.BertWeights (container layout) on `dev`."""
        gated = getattr(w, "gated", "")
        cfg = Config(num_layers=w.layers, hidden=w.hidden, num_heads=w.heads,
                     head_dim=w.head_dim, intermediate=w.ffn, vocab_size=w.vocab,
                     max_seq_len=max_seq_len, type_vocab_size=w.typ.shape[0],
                     pooling=POOL_CLS if w.cls_pool else POOL_MEAN, l2_normalize=1,
                     activation=ACT_GELU_ERF if getattr(w, "gelu_erf", False) else activation,
                     layer_norm_eps=1e-12, gated_ffn=int(bool(gated)),
                     gated_act=GATE_GELU_ERF if gated == "geglu" else GATE_SILU,
                     rope=int(getattr(w, "rope", False)),
                     rope_theta=float(getattr(w, "rope_theta", 0.0)))
        h = C.c_void_p()
        _check(lib().nebw_model_create(dev.h, C.byref(cfg), C.byref(h)))
        m = cls(dev, h)
        try:
            freq = getattr(w, "rope_inv_freq", ())
            if len(freq):  # held as float32, as the reference reads them
                f = np.ascontiguousarray(np.asarray(freq, np.float32).astype(np.float64))
                _check(lib().nebw_model_set_rope_freq(
                    m.h, f.ctypes.data_as(C.POINTER(C.c_double)), len(f)))
            for name, arr in w.tensors():
                a = np.ascontiguousarray(arr, np.float32)
                rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (1, a.shape[0])
                if name == "embeddings.position":
                    a = np.ascontiguousarray(a[:max_seq_len])
                    rows = a.shape[0]
                _check(lib().nebw_model_set_tensor(m.h, name.encode(), a.ctypes.data, F32, rows,
                                                   cols))
        except Exception:
            m.close()
            raise
        return m

    @classmethod
    def from_npue(cls, dev: Device, path):
        h = C.c_void_p()
        _check(lib().nebw_model_load_npue(dev.h, str(path).encode(), C.byref(h)))
        return cls(dev, h)

    def set_tensor(self, name: str, arr):
        """(Re)stage one tensor by its container name, fp32 (nebw_model_set_tensor)."""
        a = np.ascontiguousarray(arr, np.float32)
        rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (1, a.shape[0])
        _check(lib().nebw_model_set_tensor(self.h, name.encode(), a.ctypes.data, F32, rows, cols))

    DATAPATHS = {"bf16": 0, "i8": 1}

    def set_datapath(self, datapath: str):
        """"bf16" (default) or "i8": the int8 array path of an int8 container
        (nebw_model_set_datapath)."""
        _check(lib().nebw_model_set_datapath(self.h, self.DATAPATHS[datapath]))

    def set_graphs(self, on: bool = True):
        """encode() replays each (B, S) shape's pass as a CUDA graph (nebw_model_set_graphs)."""
        _check(lib().nebw_model_set_graphs(self.h, int(bool(on))))

    def set_int8_operand(self, name: str, kn, wscale, asmooth):
        """An int8 GEMM operand [K, N] with its .wscale [N] and .asmooth [K]."""
        q = np.ascontiguousarray(kn, np.int8)
        ws = np.ascontiguousarray(wscale, np.float32)
        asm = np.ascontiguousarray(asmooth, np.float32)
        K, N = q.shape
        _check(lib().nebw_model_set_int8_operand(self.h, name.encode(), q.ctypes.data,
                                                 ws.ctypes.data, asm.ctypes.data, K, N))

    def close(self):
        if self.h:
            lib().nebw_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def hidden(self) -> int:
        return self.cfg.hidden

    def launch_count(self, seq: int = 0) -> int:
        return lib().nebw_encode_launch_count(self.h, seq)

    KERNEL_KINDS = ("pack", "embed_ln", "gemm_qkv", "attention", "gemm_ao", "layernorm",
                    "gemm_up", "gemm_down", "pool")

    def profile(self, enable: bool = True):
        _check(lib().nebw_model_profile(self.h, int(enable)))

    def profile_collect(self) -> dict:
        """{kind: (launches, device ms)} since the last collect."""
        n = len(self.KERNEL_KINDS)
        launches = (C.c_int64 * n)()
        ms = (C.c_double * n)()
        _check(lib().nebw_model_profile_collect(self.h, launches, ms))
        return {k: (int(launches[i]), float(ms[i])) for i, k in enumerate(self.KERNEL_KINDS)}

    def encode(self, ids: np.ndarray, lens: np.ndarray) -> np.ndarray:
        """Host in, host out: ids [B, S] int32, lens [B] int32 -> [B, hidden]."""
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        B, S = ids.shape
        out = np.empty((B, self.hidden), np.float32)
        _check(lib().nebw_encode(self.h, ids.ctypes.data, lens.ctypes.data, B, S, out.ctypes.data))
        return out

    def encode_into(self, ids, lens, out, B: int, S: int, host=False, stream=None):
        """Host or device buffers by address; the device form is asynchronous."""
        if host:
            _check(lib().nebw_encode(self.h, _addr(ids), _addr(lens), B, S, _addr(out)))
        else:
            _check(lib().nebw_encode_device(self.h, _addr(ids), _addr(lens), B, S, _addr(out),
                                            _stream(stream)))


class VitModel:
    """A staged ViT encoder (container arch vit_patch16_prenorm_gelu) on one
    device: images [n, C, S, S] fp32 -> the CLS row after the final
    LayerNorm, [n, hidden] fp32."""

    KERNEL_KINDS = Model.KERNEL_KINDS

    def __init__(self, dev: Device, handle):
        self.dev = dev
        self.h = handle
        cfg = VitConfig()
        _check(lib().nebw_vit_get_config(self.h, C.byref(cfg)))
        self.cfg = cfg

    @classmethod
    def from_weights(cls, dev: Device, w):
        """Stage a nebw.synth.VitWeights on `dev`."""
        a = w.arch
        cfg = VitConfig(num_layers=w.layers, hidden=a.hidden, num_heads=a.heads,
                        head_dim=a.head_dim, intermediate=a.ffn, image_size=a.image_size,
                        patch_size=a.patch_size, num_channels=a.channels,
                        layer_norm_eps=a.ln_eps)
        h = C.c_void_p()
        _check(lib().nebw_vit_create(dev.h, C.byref(cfg), C.byref(h)))
        m = cls(dev, h)
        try:
            for name, arr in w.tensors():
                x = np.ascontiguousarray(arr, np.float32)
                rows, cols = (x.shape[0], x.shape[1]) if x.ndim == 2 else (1, x.shape[0])
                _check(lib().nebw_vit_set_tensor(m.h, name.encode(), x.ctypes.data, F32, rows,
                                                 cols))
        except Exception:
            m.close()
            raise
        return m

    @classmethod
    def from_npue(cls, dev: Device, path):
        h = C.c_void_p()
        _check(lib().nebw_vit_load_npue(dev.h, str(path).encode(), C.byref(h)))
        return cls(dev, h)

    def close(self):
        if self.h:
            lib().nebw_vit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def hidden(self) -> int:
        return self.cfg.hidden

    def launch_count(self) -> int:
        return lib().nebw_vit_launch_count(self.h)

    def profile(self, enable: bool = True):
        _check(lib().nebw_vit_profile(self.h, int(enable)))

    def profile_collect(self) -> dict:
        n = len(self.KERNEL_KINDS)
        launches = (C.c_int64 * n)()
        ms = (C.c_double * n)()
        _check(lib().nebw_vit_profile_collect(self.h, launches, ms))
        return {k: (int(launches[i]), float(ms[i])) for i, k in enumerate(self.KERNEL_KINDS)}

    def encode(self, images: np.ndarray) -> np.ndarray:
        """Host in, host out."""
        images = np.ascontiguousarray(images, np.float32)
        out = np.empty((images.shape[0], self.hidden), np.float32)
        _check(lib().nebw_vit_encode(self.h, images.ctypes.data, images.shape[0],
                                     out.ctypes.data))
        return out

    def encode_into(self, images, out, n: int, host=False, stream=None):
        """Host or device buffers by address; the device form is asynchronous."""
        if host:
            _check(lib().nebw_vit_encode(self.h, _addr(images), n, _addr(out)))
        else:
            _check(lib().nebw_vit_encode_device(self.h, _addr(images), n, _addr(out),
                                                _stream(stream)))


# ---------------------------------------------------------------------------
# several GPUs (nebw_comm): the batch sharded, the embeddings gathered
# ---------------------------------------------------------------------------

COMM_ID_BYTES = 128


def shard_plan(lens, nranks: int):
    """(owner [B], counts [nranks]) of the library's length-balanced plan."""
    lens = np.ascontiguousarray(lens, np.int32)
    owner = np.empty(len(lens), np.int32)
    counts = np.empty(nranks, np.int32)
    _check(lib().nebw_shard_plan(lens.ctypes.data, len(lens), nranks, owner.ctypes.data,
                                 counts.ctypes.data))
    return owner, counts


def shard_order(owner, nranks: int) -> np.ndarray:
    """order[k] = request index of row k of the rank-major gather."""
    owner = np.ascontiguousarray(owner, np.int32)
    order = np.empty(len(owner), np.int32)
    _check(lib().nebw_shard_order(owner.ctypes.data, len(owner), nranks, order.ctypes.data))
    return order


def comm_unique_id() -> bytes:
    buf = (C.c_uint8 * COMM_ID_BYTES)()
    _check(lib().nebw_comm_unique_id(buf))
    return bytes(buf)


class Comm:
    """A rank of an NCCL communicator on one Device (nebw_comm)."""

    def __init__(self, dev: Device, handle):
        self.dev = dev
        self.h = handle
        n, r = C.c_int32(), C.c_int32()
        _check(lib().nebw_comm_size(self.h, C.byref(n), C.byref(r)))
        self.nranks, self.rank = n.value, r.value

    @classmethod
    def init_rank(cls, dev: Device, nranks: int, rank: int, uid: bytes, timeout_s: float = 60.0):
        if len(uid) != COMM_ID_BYTES:
            raise ValueError("a communicator id is 128 bytes")
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        _check(lib().nebw_comm_init_rank(dev.h, nranks, rank, buf, timeout_s, C.byref(h)))
        return cls(dev, h)

    @classmethod
    def init_all(cls, devs, timeout_s: float = 60.0):
        n = len(devs)
        dh = (C.c_void_p * n)(*[d.h.value for d in devs])
        out = (C.c_void_p * n)()
        _check(lib().nebw_comm_init_all(n, dh, timeout_s, out))
        return [cls(d, C.c_void_p(out[i])) for i, d in enumerate(devs)]

    def close(self):
        if self.h:
            rc = lib().nebw_comm_destroy(self.h)
            self.h = None
            _check(rc)

    def __del__(self):
        try:
            if self.h:
                lib().nebw_comm_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def sync(self, stream=None):
        _check(lib().nebw_comm_sync(self.h, _stream(stream)))

    def gather_rows(self, rows, counts, H: int, out=None, root: int = 0, stream=None):
        counts = np.ascontiguousarray(counts, np.int32)
        _check(lib().nebw_gather_rows(self.h, _addr(rows), counts.ctypes.data, H, _addr(out), root,
                                      _stream(stream)))

    def encode_shard_gather(self, model: Model, ids, lens, b_r: int, S: int, counts, order=None,
                            out=None, stream=None):
        """Device-resident sharded pass (asynchronous; sync() waits)."""
        counts = np.ascontiguousarray(counts, np.int32)
        _check(lib().nebw_encode_shard_gather(model.h, self.h, _addr(ids), _addr(lens), b_r, S,
                                              counts.ctypes.data, _addr(order), _addr(out),
                                              _stream(stream)))

    def encode_sharded(self, model: Model, ids: np.ndarray, lens: np.ndarray, out=None):
        """Host buffers, synchronous; rank 0 gets [B, hidden] in request
        order (returned), the other ranks None."""
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        B, S = ids.shape
        if self.rank == 0 and out is None:
            out = np.empty((B, model.hidden), np.float32)
        _check(lib().nebw_encode_sharded(model.h, self.h, ids.ctypes.data, lens.ctypes.data, B, S,
                                         _addr(out) if self.rank == 0 else None))
        return out if self.rank == 0 else None


def encode_multi(models, comms, ids: np.ndarray, lens: np.ndarray) -> np.ndarray:
    """One process, n GPUs (Comm.init_all): [B, hidden] in request order."""
    ids = np.ascontiguousarray(ids, np.int32)
    lens = np.ascontiguousarray(lens, np.int32)
    B, S = ids.shape
    n = len(models)
    out = np.empty((B, models[0].hidden), np.float32)
    mh = (C.c_void_p * n)(*[m.h.value for m in models])
    ch = (C.c_void_p * n)(*[c.h.value for c in comms])
    _check(lib().nebw_encode_multi(n, mh, ch, ids.ctypes.data, lens.ctypes.data, B, S,
                                   out.ctypes.data))
    return out


def pack_checkpoint(model_dir, out, layout: str = "tma_bf16", max_seq: int = 0,
                    fold_scale: bool = True) -> int:
    """The library's C++ packer (nebw_pack_checkpoint); returns the bytes written."""
    n = C.c_uint64()
    _check(lib().nebw_pack_checkpoint(str(model_dir).encode(), str(out).encode(),
                                      layout.encode(), int(max_seq), int(fold_scale),
                                      C.byref(n)))
    return n.value
