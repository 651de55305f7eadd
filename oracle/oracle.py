"""TEST INFRASTRUCTURE ONLY -- Python front of the parity oracle.

Two CPU implementations of the reference's host-CPU BERT and ViT paths, both
behind ctypes:

  PortOracle  oracle/libnebw_oracle.so -- the plain-C restatement
              (oracle/bert_oracle.c).  Travels with the repository, so it is
              the checker on the GPU box.
  RefOracle   oracle/_ref/libnebw_ref.so -- the reference's own
              bert_encoder.cpp/pool.cpp/model.cpp compiled from its tree with
              its own flags (oracle/Makefile).  Built only where the
              reference tree exists; used to pin PortOracle and to make the
              golden fixtures, and as bench.py's reference arm when present.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  Nothing on the product path may.
"""

from __future__ import annotations

import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "libnebw_oracle.so"
REF_LIB = HERE / "_ref" / "libnebw_ref.so"

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_i8p = C.POINTER(C.c_int8)


def _ptr(a: np.ndarray, t=_f32p):
    return a.ctypes.data_as(t)


class _Model(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "hidden", "heads", "head_dim", "ffn",
                                          "cls_pool", "l2_normalize", "gelu_erf")] + [
        ("ln_eps", C.c_float)] + [
        (n, _f32p) for n in ("word", "pos", "typ", "emb_ln_g", "emb_ln_b")] + [
        (n, C.POINTER(_f32p)) for n in ("w_qkv", "b_qkv", "w_ao", "b_ao", "ln1_g", "ln1_b",
                                         "w_up", "b_up", "w_dn", "b_dn", "ln2_g", "ln2_b")] + [
        ("gated", C.c_int32), ("rope_inv_freq", C.POINTER(C.c_double))]


def rope_inv_freq(w) -> np.ndarray | None:
    """The rotary frequencies the reference uses for a model: its float
    list widened to double (gte, app_state.hpp:516-521), or theta^(-2j/d) in
    double (nomic, gemma_rope_tables); None for BERT."""
    if not getattr(w, "rope", False):
        return None
    if len(getattr(w, "rope_inv_freq", ())):
        return np.asarray(w.rope_inv_freq, np.float32).astype(np.float64)
    d = w.head_dim
    return np.array([1.0 / np.power(float(w.rope_theta), 2.0 * j / d) for j in range(d // 2)],
                    np.float64)


class _Vit(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "hidden", "heads", "head_dim", "ffn",
                                          "image_size", "patch_size", "channels")] + [
        ("ln_eps", C.c_float), ("attn_scale", C.c_float)] + [
        (n, _f32p) for n in ("patch_w", "patch_b", "cls", "pos", "lnf_g", "lnf_b")] + [
        (n, C.POINTER(_f32p)) for n in ("w_qkv", "b_qkv", "w_ao", "b_ao", "ln1_g", "ln1_b",
                                         "w_up", "b_up", "w_dn", "b_dn", "ln2_g", "ln2_b")]


class _I8Gemm(C.Structure):
    _fields_ = [("w", _i8p), ("ws", _f32p), ("ias", _f32p)]


def i8_operands(path, layers: int) -> dict:
    """An int8 container's GEMM operands as the array path consumes them:
    {kind: [(int8 [K, N], wscale [N], 1 / asmooth [K]) per layer]}, the panel
    untiled, the reciprocal taken in float32 as the encoder takes it
    (bert_encoder.cpp:767-772)."""
    import sys
    sys.path.insert(0, str(HERE.parent / "npu-embeddings-xdna1_b200"))
    from nebw.npue import ContainerReader, untile_block_panel  # noqa: E402
    out = {}
    with ContainerReader(path) as r:
        for g in ("qkv", "attn_out", "ffn_up", "ffn_down"):
            lst = []
            for L in range(layers):
                n = f"layer.{L}.{g}"
                e = r.entries[n]
                if e["dtype"] != "I8":
                    raise ValueError(f"{n} is {e['dtype']}, not an int8 panel")
                K, N = e["padded_shape"]
                q = untile_block_panel(np.array(r.tensor(n)).reshape(-1), K, N, e["layout"])
                ws = np.array(r.tensor(n + ".wscale"), np.float32)
                ias = (np.float32(1.0) / np.array(r.tensor(n + ".asmooth"), np.float32))
                lst.append((np.ascontiguousarray(q, np.int8), ws, ias.astype(np.float32)))
            out[g] = lst
    return out


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1




class _Int8Steps:
    """The int8 datapath's host steps, bound by symbol name: the port's
    restatement and the reference's own templates share one signature
    (quantise, dequantise, dequantise + gelu8 + quantise)."""

    _quantise = _dequantise = _dequant_gelu_quant = ""

    def _bind_int8(self):
        L = self.lib
        q = getattr(L, self._quantise)
        q.argtypes = [_f32p, C.c_int64, C.c_int64, _f32p, _i8p, _f32p]
        d = getattr(L, self._dequantise)
        d.argtypes = [_i32p, C.c_int64, C.c_int64, _f32p, _f32p, _f32p, _f32p]
        d.restype = C.c_int
        g = getattr(L, self._dequant_gelu_quant)
        g.argtypes = [_i32p, C.c_int64, C.c_int64, _f32p, _f32p, _f32p, _f32p, _i8p, _f32p]
        g.restype = C.c_int

    def quantise_rows(self, a, ias):
        a = np.ascontiguousarray(a, np.float32)
        ias = np.ascontiguousarray(ias, np.float32)
        rows, K = a.shape
        q = np.zeros((rows, K), np.int8)
        sc = np.zeros(rows, np.float32)
        getattr(self.lib, self._quantise)(_ptr(a), rows, K, _ptr(ias), _ptr(q, _i8p), _ptr(sc))
        return q, sc

    def dequantise(self, c, sa, ws, bias):
        c = np.ascontiguousarray(c, np.int32)
        sa, ws, bias = (np.ascontiguousarray(v, np.float32) for v in (sa, ws, bias))
        rows, N = c.shape
        out = np.zeros((rows, N), np.float32)
        rc = getattr(self.lib, self._dequantise)(_ptr(c, _i32p), rows, N, _ptr(sa), _ptr(ws),
                                                  _ptr(bias), _ptr(out))
        if rc:
            raise RuntimeError(f"{self._dequantise} failed ({rc})")
        return out

    def dequant_gelu_quant(self, c, sa, ws, bias, ias_next):
        c = np.ascontiguousarray(c, np.int32)
        sa, ws, bias, ias_next = (np.ascontiguousarray(v, np.float32)
                                  for v in (sa, ws, bias, ias_next))
        rows, N = c.shape
        q = np.zeros((rows, N), np.int8)
        sn = np.zeros(rows, np.float32)
        rc = getattr(self.lib, self._dequant_gelu_quant)(
            _ptr(c, _i32p), rows, N, _ptr(sa), _ptr(ws), _ptr(bias), _ptr(ias_next),
            _ptr(q, _i8p), _ptr(sn))
        if rc:
            raise RuntimeError(f"{self._dequant_gelu_quant} failed ({rc})")
        return q, sn


class PortOracle(_Int8Steps):
    """The C restatement, fed from in-memory weights."""

    _quantise = "nebw_oracle_quantise_rows"
    _dequantise = "nebw_oracle_dequantise"
    _dequant_gelu_quant = "nebw_oracle_dequant_gelu_quant"

    def __init__(self, lib_path: Path = PORT_LIB):
        if not Path(lib_path).exists():
            raise FileNotFoundError(f"{lib_path} is not built (make -C oracle port)")
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        self._bind_int8()
        L.nebw_oracle_gemm_i8.argtypes = [_i8p, C.c_int64, _i8p, C.c_int64, C.c_int64, _i32p,
                                          C.c_int32]
        L.nebw_oracle_encode.argtypes = [C.POINTER(_Model), _i32p, _i32p, C.c_int32, C.c_int32,
                                         C.c_int32, _f32p, _f32p]
        L.nebw_oracle_encode.restype = C.c_int
        L.nebw_oracle_encode_i8.argtypes = [C.POINTER(_Model)] + [C.POINTER(_I8Gemm)] * 4 + [
            _i32p, _i32p, C.c_int32, C.c_int32, C.c_int32, _f32p, _f32p]
        L.nebw_oracle_encode_i8.restype = C.c_int
        L.nebw_oracle_last_error.restype = C.c_char_p
        L.nebw_oracle_gemm_nt.argtypes = [_f32p, C.c_int64, _f32p, C.c_int64, C.c_int64, _f32p,
                                          _f32p, C.c_int32]
        L.nebw_oracle_gelu8.argtypes = [_f32p, C.c_int64]
        L.nebw_oracle_exp2.argtypes = [_f32p, C.c_int64]
        L.nebw_oracle_to_bf16.argtypes = [_f32p, C.POINTER(C.c_uint16), C.c_int64]
        L.nebw_oracle_layer_norm.argtypes = [_f32p, C.c_int64, C.c_int64, _f32p, _f32p, C.c_float]
        L.nebw_oracle_pool_rows.argtypes = [_f32p, _f32p, C.c_int64, C.c_int64, C.c_int64,
                                            C.c_int32, C.c_int32, _f32p]
        L.nebw_oracle_pool_rows.restype = C.c_int
        L.nebw_oracle_vit_encode.argtypes = [C.POINTER(_Vit), _f32p, C.c_int32, C.c_int32, _f32p,
                                             _f32p]
        L.nebw_oracle_vit_encode.restype = C.c_int
        L.nebw_oracle_vit_im2col.argtypes = [_f32p, C.c_int32, C.c_int32, C.c_int32, _f32p]

    def vit_encode(self, w, images, threads: int | None = None, hidden: bool = False):
        """ViT host path: images [n, C, S, S] -> CLS rows [n, H] (after the
        final LayerNorm); with hidden=True also every row [n, n_pos, H]."""
        a = w.arch
        images = np.ascontiguousarray(images, np.float32)
        n = images.shape[0]
        keep = []

        def arr(lst):
            v = (_f32p * len(lst))(*[_ptr(np.ascontiguousarray(x, np.float32)) for x in lst])
            keep.append(v)
            return v

        m = _Vit(layers=w.layers, hidden=a.hidden, heads=a.heads, head_dim=a.head_dim, ffn=a.ffn,
                 image_size=a.image_size, patch_size=a.patch_size, channels=a.channels,
                 ln_eps=a.ln_eps, attn_scale=1.0,
                 patch_w=_ptr(w.patch_w), patch_b=_ptr(w.patch_b), cls=_ptr(w.cls),
                 pos=_ptr(w.pos), lnf_g=_ptr(w.lnf_g), lnf_b=_ptr(w.lnf_b),
                 w_qkv=arr(w.w_qkv), b_qkv=arr(w.b_qkv), w_ao=arr(w.w_ao), b_ao=arr(w.b_ao),
                 ln1_g=arr(w.ln1_g), ln1_b=arr(w.ln1_b), w_up=arr(w.w_up), b_up=arr(w.b_up),
                 w_dn=arr(w.w_dn), b_dn=arr(w.b_dn), ln2_g=arr(w.ln2_g), ln2_b=arr(w.ln2_b))
        out = np.zeros((n, a.hidden), np.float32)
        hid = np.zeros((n, a.n_pos, a.hidden), np.float32) if hidden else None
        rc = self.lib.nebw_oracle_vit_encode(C.byref(m), _ptr(images), n,
                                             threads or host_threads(), _ptr(out),
                                             _ptr(hid) if hidden else None)
        del keep
        if rc:
            raise RuntimeError(self.lib.nebw_oracle_last_error().decode())
        return (out, hid) if hidden else out

    def vit_im2col(self, image, patch):
        image = np.ascontiguousarray(image, np.float32)
        c, s = image.shape[0], image.shape[1]
        out = np.zeros(((s // patch) ** 2, c * patch * patch), np.float32)
        self.lib.nebw_oracle_vit_im2col(_ptr(image), c, s, patch, _ptr(out))
        return out

    def _struct(self, w):
        keep = []

        def arr(lst):
            a = (_f32p * len(lst))(*[_ptr(np.ascontiguousarray(x, np.float32)) for x in lst])
            keep.append(a)
            return a

        m = _Model(layers=w.layers, hidden=w.hidden, heads=w.heads, head_dim=w.head_dim,
                   ffn=w.ffn, cls_pool=int(w.cls_pool), l2_normalize=1,
                   gelu_erf=int(getattr(w, "gelu_erf", False)), ln_eps=1e-12,
                   word=_ptr(w.word), pos=_ptr(w.pos), typ=_ptr(w.typ),
                   emb_ln_g=_ptr(w.emb_ln_g), emb_ln_b=_ptr(w.emb_ln_b),
                   w_qkv=arr(w.w_qkv), b_qkv=arr(w.b_qkv), w_ao=arr(w.w_ao), b_ao=arr(w.b_ao),
                   ln1_g=arr(w.ln1_g), ln1_b=arr(w.ln1_b), w_up=arr(w.w_up), b_up=arr(w.b_up),
                   w_dn=arr(w.w_dn), b_dn=arr(w.b_dn), ln2_g=arr(w.ln2_g), ln2_b=arr(w.ln2_b),
                   gated={"": 0, "swiglu": 1, "geglu": 2}[getattr(w, "gated", "")])
        freq = rope_inv_freq(w)
        if freq is not None:
            freq = np.ascontiguousarray(freq)
            keep.append(freq)
            m.rope_inv_freq = freq.ctypes.data_as(C.POINTER(C.c_double))
        return m, keep

    def encode(self, w, ids, mask, threads: int | None = None, hidden: bool = False):
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        B, S = ids.shape
        out = np.zeros((B, w.hidden), np.float32)
        hid = np.zeros((B * S, w.hidden), np.float32) if hidden else None
        m, keep = self._struct(w)
        rc = self.lib.nebw_oracle_encode(C.byref(m), _ptr(ids, _i32p), _ptr(mask, _i32p), B, S,
                                         threads or host_threads(), _ptr(out),
                                         _ptr(hid) if hidden else None)
        del keep
        if rc:
            raise RuntimeError(self.lib.nebw_oracle_last_error().decode())
        return (out, hid) if hidden else out

    def encode_i8(self, w, path, ids, mask, threads: int | None = None, hidden: bool = False):
        """The int8 array path (nebw_oracle_encode_i8) of the int8 container
        at `path`, packed from `w`: its GEMM operands from the container,
        embeddings, biases and LayerNorm parameters from `w` (the container
        holds them as the same fp32 values)."""
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        B, S = ids.shape
        m, keep = self._struct(w)
        ops = i8_operands(path, w.layers)
        keep.append(ops)

        def arr(kind):
            a = (_I8Gemm * w.layers)(*[_I8Gemm(_ptr(q, _i8p), _ptr(ws), _ptr(ias))
                                       for q, ws, ias in ops[kind]])
            keep.append(a)
            return a

        out = np.zeros((B, w.hidden), np.float32)
        hid = np.zeros((B * S, w.hidden), np.float32) if hidden else None
        rc = self.lib.nebw_oracle_encode_i8(C.byref(m), arr("qkv"), arr("attn_out"),
                                            arr("ffn_up"), arr("ffn_down"), _ptr(ids, _i32p),
                                            _ptr(mask, _i32p), B, S, threads or host_threads(),
                                            _ptr(out), _ptr(hid) if hidden else None)
        del keep
        if rc:
            raise RuntimeError(self.lib.nebw_oracle_last_error().decode())
        return (out, hid) if hidden else out

    def gemm_nt(self, A, B, bias, threads=1):
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        bias = np.ascontiguousarray(bias, np.float32)
        M, K = A.shape
        N = B.shape[1]
        Cm = np.zeros((M, N), np.float32)
        self.lib.nebw_oracle_gemm_nt(_ptr(A), M, _ptr(B), K, N, _ptr(bias), _ptr(Cm), threads)
        return Cm

    def gemm_i8(self, A, B, threads=1):
        """int8 [M, K] . int8 [K, N] -> int32 [M, N], exact."""
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        Cm = np.zeros((M, N), np.int32)
        self.lib.nebw_oracle_gemm_i8(_ptr(A, _i8p), M, _ptr(B, _i8p), K, N, _ptr(Cm, _i32p),
                                     threads)
        return Cm

    def gelu8(self, x):
        y = np.array(x, np.float32, copy=True)
        self.lib.nebw_oracle_gelu8(_ptr(y), y.size)
        return y

    def exp2(self, x):
        y = np.array(x, np.float32, copy=True)
        self.lib.nebw_oracle_exp2(_ptr(y), y.size)
        return y

    def to_bf16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        o = np.zeros(x.shape, np.uint16)
        self.lib.nebw_oracle_to_bf16(_ptr(x), o.ctypes.data_as(C.POINTER(C.c_uint16)), x.size)
        return o

    def layer_norm(self, x, g, b, eps=1e-12):
        y = np.array(x, np.float32, copy=True)
        self.lib.nebw_oracle_layer_norm(_ptr(y), y.shape[0], y.shape[1],
                                        _ptr(np.ascontiguousarray(g, np.float32)),
                                        _ptr(np.ascontiguousarray(b, np.float32)), eps)
        return y

    def pool_rows(self, h, am, seq, cls, l2=True):
        h = np.ascontiguousarray(h, np.float32)
        am = np.ascontiguousarray(am, np.float32)
        take = am.shape[0]
        hidden = h.shape[-1]
        out = np.zeros((take, hidden), np.float32)
        rc = self.lib.nebw_oracle_pool_rows(_ptr(h), _ptr(am), take, seq, hidden, int(cls),
                                            int(l2), _ptr(out))
        if rc:
            raise RuntimeError(self.lib.nebw_oracle_last_error().decode())
        return out


class RefOracle(_Int8Steps):
    """The reference's own host path, compiled from its tree."""

    _quantise = "nebw_ref_quantise_a_int8"
    _dequantise = "nebw_ref_dequantise_c"
    _dequant_gelu_quant = "nebw_ref_dequant_gelu_quant"

    def __init__(self, lib_path: Path = REF_LIB):
        if not Path(lib_path).exists():
            raise FileNotFoundError(f"{lib_path} is not built (make -C oracle ref)")
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        self._bind_int8()
        L.nebw_ref_encode.argtypes = [C.c_char_p, C.c_int32, _i32p, _i32p, C.c_int32, C.c_int32,
                                      _f32p, _f32p, C.c_char_p, C.c_int32]
        L.nebw_ref_encode.restype = C.c_int
        L.nebw_ref_encode_array.argtypes = L.nebw_ref_encode.argtypes
        L.nebw_ref_encode_array.restype = C.c_int
        L.nebw_ref_gemm_nt.argtypes = [_f32p, C.c_int64, _f32p, C.c_int64, C.c_int64, _f32p,
                                       _f32p, C.c_int32]
        L.nebw_ref_gelu8.argtypes = [_f32p, C.c_int64]
        L.nebw_ref_exp2.argtypes = [_f32p, C.c_int64]
        L.nebw_ref_to_bf16.argtypes = [_f32p, C.POINTER(C.c_uint16), C.c_int64]
        L.nebw_ref_pool_rows.argtypes = [_f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int32,
                                         C.c_int32, _f32p, C.c_char_p, C.c_int32]
        L.nebw_ref_pool_rows.restype = C.c_int
        L.nebw_ref_session_open.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_char_p,
                                            C.c_int32]
        L.nebw_ref_session_open.restype = C.c_void_p
        L.nebw_ref_session_run.argtypes = [C.c_void_p, _i32p, _i32p, C.c_int32, _f32p, C.c_char_p,
                                           C.c_int32]
        L.nebw_ref_session_run.restype = C.c_int
        L.nebw_ref_session_close.argtypes = [C.c_void_p]
        L.nebw_ref_vit_encode.argtypes = [C.c_char_p, _f32p, C.c_int32, C.c_int32, _f32p, _f32p,
                                          C.c_char_p, C.c_int32]
        L.nebw_ref_vit_encode.restype = C.c_int
        L.nebw_ref_vit_session_open.argtypes = [C.c_char_p, C.c_int32, C.c_char_p, C.c_int32]
        L.nebw_ref_vit_session_open.restype = C.c_void_p
        L.nebw_ref_vit_session_run.argtypes = [C.c_void_p, _f32p, C.c_int32, _f32p, C.c_char_p,
                                               C.c_int32]
        L.nebw_ref_vit_session_run.restype = C.c_int
        L.nebw_ref_vit_session_close.argtypes = [C.c_void_p]

    def vit_session(self, path, threads=None):
        """A persistent reference ViT encoder over a container (for timing)."""
        return _RefVitSession(self.lib, path, threads or host_threads())

    def vit_encode_container(self, path, images, hidden_size, n_pos=None, threads=None,
                             hidden=False):
        images = np.ascontiguousarray(images, np.float32)
        n = images.shape[0]
        out = np.zeros((n, hidden_size), np.float32)
        hid = np.zeros((n, n_pos, hidden_size), np.float32) if hidden else None
        err = C.create_string_buffer(4096)
        rc = self.lib.nebw_ref_vit_encode(str(path).encode(), _ptr(images), n,
                                          threads or host_threads(), _ptr(out),
                                          _ptr(hid) if hidden else None, err, 4096)
        if rc:
            raise RuntimeError(err.value.decode())
        return (out, hid) if hidden else out

    def vit_encode(self, w, images, threads=None, hidden=False, workdir=None):
        """Write `w` as a host-layout ViT container, then run the reference."""
        import sys
        sys.path.insert(0, str(HERE.parent / "npu-embeddings-xdna1_b200"))
        from nebw.npue import write_vit_container  # noqa: E402
        with tempfile.TemporaryDirectory(dir=workdir) as td:
            path = Path(td) / "oracle_vit.npue"
            write_vit_container(path, w)
            return self.vit_encode_container(path, images, w.arch.hidden, w.arch.n_pos,
                                             threads, hidden)

    def encode_container(self, path, seq, ids, mask, threads=None, hidden=False, hidden_size=None,
                         array=False):
        """The reference's host path on a container; with `array`, an int8
        container's array path instead (nebw_ref_encode_array: the GEMMs as
        the exact int32 products of the array, the int8 host steps around
        them)."""
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        B, S = ids.shape
        assert S == seq
        out = np.zeros((B, hidden_size), np.float32)
        hid = np.zeros((B * S, hidden_size), np.float32) if hidden else None
        err = C.create_string_buffer(4096)
        fn = self.lib.nebw_ref_encode_array if array else self.lib.nebw_ref_encode
        rc = fn(str(path).encode(), seq, _ptr(ids, _i32p), _ptr(mask, _i32p), B,
                threads or host_threads(), _ptr(out), _ptr(hid) if hidden else None, err, 4096)
        if rc:
            raise RuntimeError(err.value.decode())
        return (out, hid) if hidden else out

    def encode(self, w, ids, mask, threads=None, hidden=False, workdir=None):
        """Write `w` as a host-layout container, then run the reference."""
        import sys
        sys.path.insert(0, str(HERE.parent / "npu-embeddings-xdna1_b200"))
        from nebw.npue import write_bert_container  # noqa: E402
        S = np.asarray(ids).shape[1]
        with tempfile.TemporaryDirectory(dir=workdir) as td:
            path = Path(td) / "oracle.npue"
            write_bert_container(path, w, max_seq_len=max(S, 8))
            return self.encode_container(path, S, ids, mask, threads, hidden, w.hidden)

    def session(self, path, seq, threads=None):
        """A persistent reference encoder over a container (for timing)."""
        return _RefSession(self.lib, path, seq, threads or host_threads())

    def gemm_nt(self, A, B, bias, threads=1):
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        bias = np.ascontiguousarray(bias, np.float32)
        M, K = A.shape
        N = B.shape[1]
        Cm = np.zeros((M, N), np.float32)
        self.lib.nebw_ref_gemm_nt(_ptr(A), M, _ptr(B), K, N, _ptr(bias), _ptr(Cm), threads)
        return Cm

    def gelu8(self, x):
        y = np.array(x, np.float32, copy=True)
        self.lib.nebw_ref_gelu8(_ptr(y), y.size)
        return y

    def exp2(self, x):
        y = np.array(x, np.float32, copy=True)
        self.lib.nebw_ref_exp2(_ptr(y), y.size)
        return y

    def to_bf16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        o = np.zeros(x.shape, np.uint16)
        self.lib.nebw_ref_to_bf16(_ptr(x), o.ctypes.data_as(C.POINTER(C.c_uint16)), x.size)
        return o

    def pool_rows(self, h, am, seq, cls, l2=True):
        h = np.ascontiguousarray(h, np.float32)
        am = np.ascontiguousarray(am, np.float32)
        take = am.shape[0]
        hidden = h.shape[-1]
        out = np.zeros((take, hidden), np.float32)
        err = C.create_string_buffer(1024)
        rc = self.lib.nebw_ref_pool_rows(_ptr(h), _ptr(am), take, seq, hidden, int(cls), int(l2),
                                         _ptr(out), err, 1024)
        if rc:
            raise RuntimeError(err.value.decode())
        return out


class _RefSession:
    def __init__(self, lib, path, seq, threads):
        self.lib, self.seq, self.threads = lib, seq, threads
        err = C.create_string_buffer(4096)
        self.h = lib.nebw_ref_session_open(str(path).encode(), seq, threads, err, 4096)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def run(self, ids, mask, hidden_size):
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        assert ids.shape[1] == self.seq
        out = np.zeros((ids.shape[0], hidden_size), np.float32)
        err = C.create_string_buffer(4096)
        if self.lib.nebw_ref_session_run(self.h, _ptr(ids, _i32p), _ptr(mask, _i32p), ids.shape[0],
                                         _ptr(out), err, 4096):
            raise RuntimeError(err.value.decode())
        return out

    def close(self):
        if self.h:
            self.lib.nebw_ref_session_close(self.h)
            self.h = None


class _RefVitSession:
    def __init__(self, lib, path, threads):
        self.lib = lib
        err = C.create_string_buffer(4096)
        self.h = lib.nebw_ref_vit_session_open(str(path).encode(), threads, err, 4096)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def run(self, images, hidden_size):
        images = np.ascontiguousarray(images, np.float32)
        out = np.zeros((images.shape[0], hidden_size), np.float32)
        err = C.create_string_buffer(4096)
        if self.lib.nebw_ref_vit_session_run(self.h, _ptr(images), images.shape[0], _ptr(out),
                                             err, 4096):
            raise RuntimeError(err.value.decode())
        return out

    def close(self):
        if self.h:
            self.lib.nebw_ref_vit_session_close(self.h)
            self.h = None

    def __del__(self):
        self.close()
