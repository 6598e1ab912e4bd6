"""ctypes bindings for the CPU checker (oracle/liboracle.so) and for the
reference's own code built in place (oracle/_ref/libref_moe.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, never by the product package.
"""
from __future__ import annotations

import ctypes as C  # noqa: N812
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref_moe.so")
REF_GGUF_PATH = os.path.join(HERE, "_ref", "libref_gguf.so")

TYPE_F32 = 0
TYPE_F16 = 1
TYPE_BF16 = 30
TYPE_Q4_K = 12
TYPE_Q6_K = 14
QK = 256
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210}
# synthetic tensor kinds (stream ids), shared with the CUDA library's generator
KIND_GATE, KIND_UP, KIND_DOWN, KIND_ROUTER, KIND_BIAS, KIND_NORM, KIND_ACT = range(7)

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build():
    """Compile the checker (and the reference, when its sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class LayerCfg(C.Structure):
    _fields_ = [("H", C.c_int), ("I", C.c_int), ("n_experts", C.c_int), ("n_group", C.c_int),
                ("topk_group", C.c_int), ("K", C.c_int), ("routed_scale", C.c_float),
                ("down_type", C.c_int)]


class MlaCfg(C.Structure):
    _fields_ = [("H", C.c_int), ("n_heads", C.c_int), ("q_lora", C.c_int), ("kv_lora", C.c_int),
                ("qk_nope", C.c_int), ("qk_rope", C.c_int), ("v_head", C.c_int), ("rope_theta", C.c_float),
                ("rope_scale", C.c_float), ("rope_orig_ctx", C.c_float), ("eps", C.c_float)]


class MlaWeights(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("q_a", "q_b", "kv_a", "k_b", "v_b", "o_proj", "attn_norm", "q_a_norm",
                                          "kv_a_norm")]


# DeepSeek-V3 / R1 attention shapes (infer.m:44-65)
MLA_DEEPSEEK = dict(H=7168, n_heads=128, q_lora=1536, kv_lora=512, qk_nope=128, qk_rope=64, v_head=128,
                    rope_theta=10000.0, rope_scale=40.0, rope_orig_ctx=4096.0, eps=1e-6)

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.or_fp16_to_fp32.restype = C.c_float
        L.or_fp16_to_fp32.argtypes = [C.c_uint16]
        L.or_fp32_to_fp16.restype = C.c_uint16
        L.or_fp32_to_fp16.argtypes = [C.c_float]
        for fn in (L.or_dequant_q4k, L.or_dequant_q6k):
            fn.restype = None
            fn.argtypes = [_u8p, _f32p, C.c_size_t]
        L.or_quantize_q4k.argtypes = [_f32p, _u8p, C.c_size_t]
        L.or_quantize_q6k.argtypes = [_f32p, _u8p, C.c_size_t]
        L.or_splitmix64.restype = C.c_uint64
        L.or_splitmix64.argtypes = [C.c_uint64]
        L.or_stream.restype = C.c_uint64
        L.or_stream.argtypes = [C.c_int, C.c_int, C.c_int]
        L.or_det_log.restype = C.c_double
        L.or_det_log.argtypes = [C.c_double]
        L.or_normal.restype = C.c_double
        L.or_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        L.or_fill_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_size_t, C.c_double, _f32p, C.c_int]
        L.or_gen_matrix.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_double, _u8p, C.c_int]
        L.or_sigmoidf.restype = C.c_float
        L.or_sigmoidf.argtypes = [C.c_float]
        L.or_silu_mul.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        L.or_rms_norm.argtypes = [_f32p, C.c_void_p, _f32p, C.c_int, C.c_float]
        L.or_route.argtypes = [_f32p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _i32p, _f32p]
        L.or_qmatvec.argtypes = [_u8p, C.c_int, C.c_int, C.c_int, _f32p, _f32p, C.c_int, C.c_int]
        L.or_router_logits.argtypes = [_f32p, _f32p, C.c_int, C.c_int, _f32p, C.c_int]
        L.or_expert_forward.argtypes = [_u8p, _u8p, _u8p, C.c_int, _f32p, C.c_int, C.c_int, _f32p, C.c_int, C.c_int]
        L.or_expert_bytes.restype = C.c_size_t
        L.or_expert_bytes.argtypes = [C.c_int, C.c_int, C.c_int]
        L.or_moe_layer.argtypes = [C.POINTER(LayerCfg), C.POINTER(C.c_void_p), _f32p, C.c_void_p, _f32p, C.c_int,
                                   C.c_void_p, C.c_void_p, _f32p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_int, C.c_int]
        L.or_moe_layer_given.argtypes = [C.POINTER(LayerCfg), C.POINTER(C.c_void_p), _f32p, C.c_int, _i32p, _f32p,
                                         _f32p, C.c_int, C.c_int]
        _u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        L.or_to_f16.restype = C.c_int
        L.or_to_f16.argtypes = [C.c_int, C.c_void_p, _u16p, C.c_size_t]
        L.or_mv_f16.argtypes = [_u16p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.or_dense_ffn.argtypes = [_u16p, _u16p, _u16p, C.c_int, C.c_int, _f32p, C.c_int, _f32p, C.c_int, C.c_int]
        L.or_argmax.restype = C.c_int
        L.or_argmax.argtypes = [_f32p, C.c_int]
        L.or_rand_unit.restype = C.c_float
        L.or_rand_unit.argtypes = [C.POINTER(C.c_uint32)]
        L.or_sample_top_p.restype = C.c_int
        L.or_sample_top_p.argtypes = [_f32p, C.c_int, C.c_float, C.c_float, C.POINTER(C.c_uint32),
                                      C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.or_yarn_band.argtypes = [C.POINTER(MlaCfg), C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.or_yarn_freq.restype = C.c_float
        L.or_yarn_freq.argtypes = [C.POINTER(MlaCfg), C.c_int]
        L.or_rope.argtypes = [C.POINTER(MlaCfg), _f32p, C.c_int, C.c_int]
        L.or_softmax.argtypes = [_f32p, C.c_int]
        L.or_mla_decode.argtypes = [C.POINTER(MlaCfg), C.POINTER(MlaWeights), _f32p, _f32p, _f32p,
                                    C.POINTER(C.c_int), C.c_int, C.c_int]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own quant.c / route() / silu_mul / rms_norm / argmax /
    sample_top_p."""
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        R.fp16_to_fp32.restype = C.c_float
        R.fp16_to_fp32.argtypes = [C.c_uint16]
        R.dequantize_row_q4_K.argtypes = [_u8p, _f32p, C.c_size_t]
        R.dequantize_row_q6_K.argtypes = [_u8p, _f32p, C.c_size_t]
        R.ref_sigmoidf.restype = C.c_float
        R.ref_sigmoidf.argtypes = [C.c_float]
        R.ref_silu_mul.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        R.ref_rms_norm.argtypes = [_f32p, C.c_void_p, _f32p, C.c_int]
        R.ref_route.argtypes = [_f32p, C.c_void_p, C.c_int, _i32p, _f32p]
        R.ref_moe_token_cpu.restype = C.c_int
        R.ref_moe_token_cpu.argtypes = [C.POINTER(C.c_void_p), C.c_int, _f32p, _f32p, _f32p, _f32p, C.c_int,
                                        _f32p, C.c_void_p, C.c_void_p, C.c_int]
        R.ref_argmax.restype = C.c_int
        R.ref_argmax.argtypes = [_f32p, C.c_int]
        R.ref_sample_top_p.restype = C.c_int
        R.ref_sample_top_p.argtypes = [_f32p, C.c_int, C.c_float, C.c_float, C.POINTER(C.c_uint32)]
        R.ref_softmax.argtypes = [_f32p, C.c_int]
        R.ref_yarn_freq.restype = C.c_float
        R.ref_yarn_freq.argtypes = [C.c_int]
        R.ref_yarn_band.argtypes = [C.POINTER(C.c_int), C.POINTER(C.c_int)]
        R.ref_rope_q.argtypes = [_f32p, C.c_int, C.c_int]
        R.ref_rope_k.argtypes = [_f32p, C.c_int]
        _ref = R
    return _ref


def ref_gguf_available() -> bool:
    return os.path.exists(REF_GGUF_PATH)


def ref_gguf_tensor(path: str, name: str):
    """(dims, ggml type, bytes) of tensor `name` in the GGUF file at `path`,
    read by the reference's own gguf.c (gguf_load_manifest / gguf_find /
    gguf_tensor_pread, gguf.h:168-192); None if the tensor is absent."""
    R = C.CDLL(REF_GGUF_PATH)
    R.ref_gguf_tensor.restype = C.c_int
    R.ref_gguf_tensor.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint32),
                                  C.POINTER(C.c_int), C.POINTER(C.c_uint64), C.c_void_p, C.c_uint64]
    dims = (C.c_uint64 * 4)()
    nd, ty, nb = C.c_uint32(), C.c_int(), C.c_uint64()
    rc = R.ref_gguf_tensor(path.encode(), name.encode(), dims, C.byref(nd), C.byref(ty), C.byref(nb), None, 0)
    if rc == -2:
        return None
    if rc != 0:
        raise RuntimeError(f"gguf.c could not read {path} ({rc})")
    buf = np.empty(nb.value, np.uint8)
    rc = R.ref_gguf_tensor(path.encode(), name.encode(), dims, C.byref(nd), C.byref(ty), C.byref(nb),
                           buf.ctypes.data, buf.size)
    if rc != 0:
        raise RuntimeError(f"gguf.c could not read {name} ({rc})")
    return [int(dims[i]) for i in range(nd.value)], ty.value, buf


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- wrappers
def row_bytes(qtype: int, cols: int) -> int:
    return cols // QK * BLOCK_BYTES[qtype]


def dequant(blob: np.ndarray, qtype: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    b = np.ascontiguousarray(blob, dtype=np.uint8)
    (lib().or_dequant_q6k if qtype == TYPE_Q6_K else lib().or_dequant_q4k)(b, out, n)
    return out


def ref_dequant(blob: np.ndarray, qtype: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    b = np.ascontiguousarray(blob, dtype=np.uint8)
    (ref().dequantize_row_q6_K if qtype == TYPE_Q6_K else ref().dequantize_row_q4_K)(b, out, n)
    return out


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size // QK * BLOCK_BYTES[qtype], np.uint8)
    (lib().or_quantize_q6k if qtype == TYPE_Q6_K else lib().or_quantize_q4k)(x, out, x.size)
    return out


def stream(layer: int, expert: int, kind: int) -> int:
    return lib().or_stream(layer, expert, kind)


def normal(seed: int, strm: int, n: int, sigma: float = 1.0, first: int = 0, threads: int = 8) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_fill_normal(seed, strm, first, n, sigma, out, threads)
    return out


def gen_matrix(seed: int, strm: int, qtype: int, rows: int, cols: int, sigma: float, threads: int = 8):
    out = np.empty(rows * row_bytes(qtype, cols), np.uint8)
    lib().or_gen_matrix(seed, strm, qtype, rows, cols, sigma, out, threads)
    return out


def gen_expert(seed: int, layer: int, expert: int, H: int, I: int, down_type: int, sigma: float = 0.02,
               threads: int = 8) -> np.ndarray:
    """[gate Q4_K][up Q4_K][down] blob of one synthetic expert."""
    g = gen_matrix(seed, stream(layer, expert, KIND_GATE), TYPE_Q4_K, I, H, sigma, threads)
    u = gen_matrix(seed, stream(layer, expert, KIND_UP), TYPE_Q4_K, I, H, sigma, threads)
    d = gen_matrix(seed, stream(layer, expert, KIND_DOWN), down_type, H, I, sigma, threads)
    return np.concatenate([g, u, d])


def expert_bytes(H: int, I: int, down_type: int) -> int:
    return lib().or_expert_bytes(H, I, down_type)


def route(logits, bias, n_group=8, topk_group=4, K=8, scale=2.5):
    logits = np.ascontiguousarray(logits, np.float32)
    E = logits.size
    idx = np.zeros(K, np.int32)
    w = np.zeros(K, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().or_route(logits, _ptr(b), E, n_group, topk_group, K, scale, idx, w)
    return idx, w


def ref_route(logits, bias, K=8):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.zeros(K, np.int32)
    w = np.zeros(K, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ref().ref_route(logits, _ptr(b), K, idx, w)
    return idx, w


def qmatvec(W, qtype, rows, cols, x, acc_double=True, threads=8):
    y = np.empty(rows, np.float32)
    lib().or_qmatvec(np.ascontiguousarray(W, np.uint8), qtype, rows, cols,
                     np.ascontiguousarray(x, np.float32), y, int(acc_double), threads)
    return y


def expert_forward(blob, H, I, down_type, x, acc_double=True, threads=8):
    gb = row_bytes(TYPE_Q4_K, H) * I
    blob = np.ascontiguousarray(blob, np.uint8)
    eo = np.empty(H, np.float32)
    lib().or_expert_forward(blob[:gb], blob[gb:2 * gb], blob[2 * gb:], down_type,
                            np.ascontiguousarray(x, np.float32), H, I, eo, int(acc_double), threads)
    return eo


def to_f16(blob, qtype: int, n: int) -> np.ndarray:
    """A GGUF tensor of n values (F32, F16, BF16, Q4_K, Q6_K) as fp16 bits,
    the way the reference keeps its dense FFN weights."""
    b = np.ascontiguousarray(blob).view(np.uint8).reshape(-1)
    out = np.empty(n, np.uint16)
    if lib().or_to_f16(qtype, b.ctypes.data_as(C.c_void_p), out, n) != 0:
        raise ValueError(f"type {qtype} not decodable to fp16")
    return out


def mv_f16(A, x, acc_double=True, threads=8):
    A = np.ascontiguousarray(A, np.uint16)
    m, n = A.shape
    y = np.empty(m, np.float32)
    lib().or_mv_f16(A, np.ascontiguousarray(x, np.float32), y, m, n, int(acc_double), threads)
    return y


def dense_ffn(gate, up, down, x, acc_double=True, threads=8):
    """gate, up: fp16 bits [Id x H]; down: fp16 bits [H x Id]; x [T x H]."""
    Id, H = gate.shape
    x = np.ascontiguousarray(x, np.float32).reshape(-1, H)
    out = np.empty_like(x)
    lib().or_dense_ffn(np.ascontiguousarray(gate, np.uint16), np.ascontiguousarray(up, np.uint16),
                       np.ascontiguousarray(down, np.uint16), H, Id, x, x.shape[0], out, int(acc_double), threads)
    return out


def sample_top_p(logits, temp: float, top_p: float, state: int):
    """(token, next state, nucleus mass, draw) of one row, as infer.m:419-456."""
    st = C.c_uint32(state)
    cum, r = C.c_float(0), C.c_float(0)
    lg = np.ascontiguousarray(logits, np.float32)
    tok = lib().or_sample_top_p(lg, lg.size, temp, top_p, C.byref(st), C.byref(cum), C.byref(r))
    return tok, st.value, cum.value, r.value


def mla_cfg(**kw) -> MlaCfg:
    d = dict(MLA_DEEPSEEK)
    d.update(kw)
    return MlaCfg(**d)


class MlaCache:
    """The per-layer latent cache of mla_forward (MLACache, infer.m:665-675)."""

    def __init__(self, cfg: MlaCfg, max_seq: int):
        self.c_kv = np.zeros((max_seq, cfg.kv_lora), np.float32)
        self.k_rope = np.zeros((max_seq, cfg.qk_rope), np.float32)
        self.len = 0


def mla_decode(cfg: MlaCfg, w: dict, hidden, cache: MlaCache, pos: int, acc_double=True):
    """hidden + attention of one token (infer.m:766-903); w holds fp16-bit
    matrices q_a, q_b, kv_a, k_b, v_b, o_proj and fp32 norms attn_norm,
    q_a_norm, kv_a_norm; the cache gains one row."""
    arrs = {k: np.ascontiguousarray(w[k], np.uint16) for k in ("q_a", "q_b", "kv_a", "k_b", "v_b", "o_proj")}
    arrs.update({k: np.ascontiguousarray(w[k], np.float32) for k in ("attn_norm", "q_a_norm", "kv_a_norm")})
    ws = MlaWeights(**{k: a.ctypes.data for k, a in arrs.items()})
    h = np.array(hidden, np.float32, copy=True).reshape(-1)
    n = C.c_int(cache.len)
    lib().or_mla_decode(C.byref(cfg), C.byref(ws), h, cache.c_kv, cache.k_rope, C.byref(n), pos, int(acc_double))
    cache.len = n.value
    return h


def moe_layer(cfg: dict, experts: dict, router_w, bias, x, force_idx=None, force_w=None,
              acc_double=True, threads=8):
    """experts: {expert_id: blob}; only the ids the routing touches (and the
    shared expert, id n_experts) need to be present."""
    E = cfg["n_experts"]
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cfg["H"])
    B = x.shape[0]
    c = LayerCfg(cfg["H"], cfg["I"], E, cfg["n_group"], cfg["topk_group"], cfg["K"],
                 cfg["routed_scale"], cfg["down_type"])
    table = (C.c_void_p * (E + 1))()
    keep = []
    for e, blob in experts.items():
        blob = np.ascontiguousarray(blob, np.uint8)
        keep.append(blob)
        table[e] = blob.ctypes.data
    out = np.empty((B, cfg["H"]), np.float32)
    idx = np.empty((B, cfg["K"]), np.int32)
    w = np.empty((B, cfg["K"]), np.float32)
    logits = np.empty((B, E), np.float32)
    fi = None if force_idx is None else np.ascontiguousarray(force_idx, np.int32)
    fw = None if force_w is None else np.ascontiguousarray(force_w, np.float32)
    lib().or_moe_layer(C.byref(c), table, np.ascontiguousarray(router_w, np.float32),
                       _ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)), x, B,
                       _ptr(fi), _ptr(fw), out, _ptr(idx), _ptr(w), _ptr(logits), int(acc_double), threads)
    return out, idx, w, logits


def moe_layer_given(cfg: dict, experts: dict, x, idx, w, acc_double=True, threads=None):
    """The layer's output for a batch whose routing is given, grouped by
    expert (each weight row dequantized once per expert): identical, bit for
    bit, to moe_layer(..., force_idx=idx, force_w=w), and much faster for
    many tokens.  experts: {expert_id: blob} for every routed id and the
    shared expert (id n_experts)."""
    if threads is None:
        threads = max(1, len(os.sched_getaffinity(0)))
    E = cfg["n_experts"]
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cfg["H"])
    B = x.shape[0]
    c = LayerCfg(cfg["H"], cfg["I"], E, cfg["n_group"], cfg["topk_group"], cfg["K"],
                 cfg["routed_scale"], cfg["down_type"])
    table = (C.c_void_p * (E + 1))()
    keep = []
    for e, blob in experts.items():
        blob = np.ascontiguousarray(blob, np.uint8)
        keep.append(blob)
        table[e] = blob.ctypes.data
    out = np.empty((B, cfg["H"]), np.float32)
    lib().or_moe_layer_given(C.byref(c), table, x, B, np.ascontiguousarray(idx, np.int32),
                             np.ascontiguousarray(w, np.float32), out, int(acc_double), threads)
    return out
