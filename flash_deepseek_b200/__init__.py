"""flash_deepseek_b200 -- the DeepSeek-V3/R1 mixture-of-experts block on NVIDIA
B200 (sm_100a), behind the C ABI of libmoe_cuda.so.

This module is the Python mirror of that ABI, named after the reference
engine's own seams (JohnnyNg6/flash_deepseek, infer.m):

    MoE.route            route()                infer.m:920-991
    MoE.experts_forward  metal_moe_forward()    infer.m:1604-1700
    MoE.shared_forward   shared_expert_worker() infer.m:1099-1114
    MoE.forward          MoE half of layer_forward, infer.m:1878-1922
    dequantize_row_q4_K / dequantize_row_q6_K   quant.h:11-12

Host arrays are numpy; device buffers may be given as integer pointers or as
objects with ``data_ptr()`` (torch tensors).  All compute runs in the CUDA
library; if it is missing, importing ``load_library`` raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

from ._lib import MoeConfigC, load as load_library

TYPE_F32 = 0  # GGML_TYPE_F32
TYPE_F16 = 1  # GGML_TYPE_F16
TYPE_Q4_K = 12  # GGML_TYPE_Q4_K (gguf.h:59)
TYPE_Q6_K = 14  # GGML_TYPE_Q6_K (gguf.h:61)
TYPE_BF16 = 30  # GGML_TYPE_BF16
QK_K = 256
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210}


class MoeError(RuntimeError):
    pass


@dataclass
class MoeConfig:
    """Model constants of infer.m:43-80 (DeepSeek-V3/R1 defaults)."""
    hidden: int = 7168
    intermediate: int = 2048
    n_experts: int = 256
    n_group: int = 8
    topk_group: int = 4
    top_k: int = 8
    routed_scale: float = 2.5
    rms_eps: float = 1e-6
    n_layers: int = 1
    max_tokens: int = 64

    def c(self) -> MoeConfigC:
        return MoeConfigC(self.hidden, self.intermediate, self.n_experts, self.n_group, self.topk_group,
                          self.top_k, self.routed_scale, self.rms_eps, self.n_layers, self.max_tokens)


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays passed to the CUDA library must be C-contiguous")
        return a.ctypes.data
    raise TypeError(f"cannot pass {type(a)} as a pointer")


def _f32(a, shape=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a if shape is None else a.reshape(shape)


def row_bytes(qtype: int, cols: int) -> int:
    return cols // QK_K * BLOCK_BYTES[qtype]


def get_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    rc = load_library().moe_get_unique_id(C.cast(buf, C.c_void_p))
    if rc != 0:
        raise MoeError(f"moe_get_unique_id failed ({rc})")
    return bytes(buf)


class MoE:
    """One context of libmoe_cuda.so on one GPU (one per rank for expert
    parallelism)."""

    def __init__(self, cfg: MoeConfig, device: int = 0, rank: int = 0, world_size: int = 1,
                 unique_id: bytes | None = None):
        self.lib = load_library()
        self.cfg = cfg
        self._c = cfg.c()
        uid = None
        if unique_id is not None:
            self._uid = (C.c_ubyte * 128).from_buffer_copy(unique_id)
            uid = C.cast(self._uid, C.c_void_p)
        self.ctx = self.lib.moe_create(C.byref(self._c), device, rank, world_size, uid)
        if not self.ctx:
            raise MoeError("moe_create failed (see stderr)")
        self.rank, self.world_size, self.device = rank, world_size, device

    # -------------------------------------------------------------- plumbing
    def close(self):
        if getattr(self, "ctx", None):
            self.lib.moe_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self.lib.moe_last_error(self.ctx)
            raise MoeError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")

    @property
    def stream(self) -> int:
        return self.lib.moe_stream(self.ctx) or 0

    @property
    def kernel_launches(self) -> int:
        return int(self.lib.moe_kernel_launches(self.ctx))

    def reset_kernel_launches(self):
        self.lib.moe_reset_kernel_launches(self.ctx)

    def last_weight_bytes(self) -> int:
        return int(self.lib.moe_last_weight_bytes(self.ctx))

    @property
    def ep_peer_memory(self) -> bool:
        """True when the expert-parallel exchanges run over NVLink peer memory."""
        return bool(self.lib.moe_ep_peer_memory(self.ctx))

    def record_expert_hits(self, d_hits):
        """While d_hits (device int32 [n_layers]) is set, every device forward
        writes d_hits[layer] = routed experts of this rank hit by that layer;
        None stops recording."""
        self._check(self.lib.moe_record_expert_hits(self.ctx, _ptr(d_hits)), "moe_record_expert_hits")

    def set_timing(self, ring_steps: int = 1):
        """Record per-phase CUDA events for the last `ring_steps` forward calls
        (0 turns timing off)."""
        self._check(self.lib.moe_set_timing(self.ctx, int(ring_steps)), "moe_set_timing")

    def timing(self, back: int = 0) -> dict:
        """Per-phase device milliseconds of the `back`-th most recent call."""
        from ._lib import PHASES
        ms = (C.c_float * len(PHASES))()
        self._check(self.lib.moe_get_timing_at(self.ctx, back, C.cast(ms, C.c_void_p), len(PHASES)),
                    "moe_get_timing_at")
        return dict(zip(PHASES, list(ms)))

    # --------------------------------------------------------------- weights
    def load_layer(self, layer, gate_exps, up_exps, down_exps, down_type, router_w, bias, sh_gate, sh_up, sh_down,
                   sh_down_type):
        arrs = [np.ascontiguousarray(a, np.uint8) for a in (gate_exps, up_exps, down_exps, sh_gate, sh_up, sh_down)]
        rw = _f32(router_w)
        b = None if bias is None else _f32(bias)
        self._check(self.lib.moe_load_layer(self.ctx, layer, _ptr(arrs[0]), _ptr(arrs[1]), _ptr(arrs[2]), down_type,
                                            _ptr(rw), _ptr(b), _ptr(arrs[3]), _ptr(arrs[4]), _ptr(arrs[5]),
                                            sh_down_type), "moe_load_layer")

    def shard_range(self, per_expert_bytes: int) -> tuple[int, int]:
        """(offset, bytes) of this rank's experts inside a stacked expert tensor."""
        off, n = C.c_size_t(), C.c_size_t()
        self._check(self.lib.moe_shard_range(self.ctx, per_expert_bytes, C.byref(off), C.byref(n)),
                    "moe_shard_range")
        return off.value, n.value

    def load_layer_shard(self, layer, gate_slice, up_slice, down_slice, down_type, router_w, bias, sh_gate, sh_up,
                         sh_down, sh_down_type):
        """moe_load_layer with the expert tensors cut to this rank's slice."""
        arrs = [np.ascontiguousarray(a, np.uint8) for a in (gate_slice, up_slice, down_slice, sh_gate, sh_up, sh_down)]
        rw = _f32(router_w)
        b = None if bias is None else _f32(bias)
        self._check(self.lib.moe_load_layer_shard(self.ctx, layer, _ptr(arrs[0]), _ptr(arrs[1]), _ptr(arrs[2]),
                                                  down_type, _ptr(rw), _ptr(b), _ptr(arrs[3]), _ptr(arrs[4]),
                                                  _ptr(arrs[5]), sh_down_type), "moe_load_layer_shard")

    def write_layer_packed(self, layer: int, path: str):
        """This rank's experts of `layer` into the reference's packed layer file."""
        self._check(self.lib.moe_write_layer_packed(self.ctx, layer, os.fsencode(path)), "moe_write_layer_packed")

    def load_layer_packed(self, layer, layer_blob, expert_size, router_w, bias, sh_gate, sh_up, sh_down,
                          sh_down_type):
        blob = np.ascontiguousarray(layer_blob, np.uint8)
        sh = [np.ascontiguousarray(a, np.uint8) for a in (sh_gate, sh_up, sh_down)]
        rw = _f32(router_w)
        b = None if bias is None else _f32(bias)
        self._check(self.lib.moe_load_layer_packed(self.ctx, layer, _ptr(blob), expert_size, _ptr(rw), _ptr(b),
                                                   _ptr(sh[0]), _ptr(sh[1]), _ptr(sh[2]), sh_down_type),
                    "moe_load_layer_packed")

    def init_layer_synthetic(self, layer: int, seed: int = 0, down_type: int = TYPE_Q6_K, w_sigma: float = 0.02,
                             router_sigma: float = 0.006, bias_sigma: float = 0.01):
        self._check(self.lib.moe_init_layer_synthetic(self.ctx, layer, seed, down_type, w_sigma, router_sigma,
                                                      bias_sigma), "moe_init_layer_synthetic")

    def add_router_bias(self, layer: int, extra_bias):
        eb = _f32(extra_bias)
        self._check(self.lib.moe_add_router_bias(self.ctx, layer, _ptr(eb)), "moe_add_router_bias")

    def set_logit_bias(self, layer: int, logit_bias):
        """Per-expert term added to the router logits before the sigmoid (None
        clears it)."""
        lb = None if logit_bias is None else _f32(logit_bias)
        self._check(self.lib.moe_set_logit_bias(self.ctx, layer, _ptr(lb)), "moe_set_logit_bias")

    def set_norm_weight(self, layer: int, w):
        w = _f32(w)
        self._check(self.lib.moe_set_norm_weight(self.ctx, layer, _ptr(w)), "moe_set_norm_weight")

    def expert_bytes(self, layer: int) -> int:
        return int(self.lib.moe_expert_bytes(self.ctx, layer))

    def read_expert(self, layer: int, expert: int) -> np.ndarray:
        n = self.expert_bytes(layer)
        if expert == self.cfg.n_experts:  # the shared expert may have another down type
            n = max(n, 2 * row_bytes(TYPE_Q4_K, self.cfg.hidden) * self.cfg.intermediate +
                    row_bytes(TYPE_Q6_K, self.cfg.intermediate) * self.cfg.hidden)
        out = np.empty(n, np.uint8)
        self._check(self.lib.moe_read_expert(self.ctx, layer, expert, _ptr(out), n), "moe_read_expert")
        return out

    # ------------------------------------------------------ dense FFN layers
    def load_dense_layer(self, layer: int, gate, gate_type: int, up, up_type: int, down, down_type: int,
                         intermediate: int):
        """The dense FFN of a first layer (infer.m:1786-1793) from GGUF bytes
        (numpy arrays of any dtype, read as raw bytes)."""
        bufs = [np.ascontiguousarray(b).view(np.uint8) for b in (gate, up, down)]
        self._check(self.lib.moe_load_dense_layer(self.ctx, layer, intermediate, _ptr(bufs[0]), gate_type,
                                                  _ptr(bufs[1]), up_type, _ptr(bufs[2]), down_type),
                    "moe_load_dense_layer")

    def init_dense_synthetic(self, layer: int, intermediate: int, seed: int = 0, w_sigma: float = 0.02):
        self._check(self.lib.moe_init_dense_synthetic(self.ctx, layer, intermediate, seed, w_sigma),
                    "moe_init_dense_synthetic")

    def read_dense_weight(self, layer: int, which: int, intermediate: int) -> np.ndarray:
        """Matrix `which` (0 gate, 1 up, 2 down) as fp16 bits (uint16)."""
        out = np.empty(intermediate * self.cfg.hidden, np.uint16)
        self._check(self.lib.moe_read_dense_weight(self.ctx, layer, which, _ptr(out), out.nbytes),
                    "moe_read_dense_weight")
        return out.reshape((intermediate, self.cfg.hidden) if which < 2 else (self.cfg.hidden, intermediate))

    def dense_forward(self, layer: int, h_post):
        h = _f32(h_post).reshape(-1, self.cfg.hidden)
        out = np.empty_like(h)
        self._check(self.lib.moe_dense_forward(self.ctx, layer, _ptr(h), h.shape[0], _ptr(out)),
                    "moe_dense_forward")
        return out

    def dense_forward_device(self, layer: int, d_h, n_tokens: int, d_out, stream=None):
        self._check(self.lib.moe_dense_forward_device(self.ctx, layer, _ptr(d_h), n_tokens, _ptr(d_out),
                                                      _ptr(stream)), "moe_dense_forward_device")

    # ------------------------------------------------- output head, sampling
    def load_lm_head(self, w, qtype: int, vocab: int):
        b = np.ascontiguousarray(w).view(np.uint8)
        self._check(self.lib.moe_load_lm_head(self.ctx, vocab, _ptr(b), qtype), "moe_load_lm_head")
        self.vocab = vocab

    def init_lm_head_synthetic(self, vocab: int, seed: int = 0, w_sigma: float = 0.02):
        self._check(self.lib.moe_init_lm_head_synthetic(self.ctx, vocab, seed, w_sigma), "moe_init_lm_head_synthetic")
        self.vocab = vocab

    def read_lm_head(self) -> np.ndarray:
        out = np.empty((self.vocab, self.cfg.hidden), np.uint16)
        self._check(self.lib.moe_read_lm_head(self.ctx, _ptr(out), out.nbytes), "moe_read_lm_head")
        return out

    def lm_head(self, h):
        h = _f32(h).reshape(-1, self.cfg.hidden)
        out = np.empty((h.shape[0], self.vocab), np.float32)
        self._check(self.lib.moe_lm_head(self.ctx, _ptr(h), h.shape[0], _ptr(out)), "moe_lm_head")
        return out

    def lm_head_device(self, d_h, n_tokens: int, d_logits, stream=None):
        self._check(self.lib.moe_lm_head_device(self.ctx, _ptr(d_h), n_tokens, _ptr(d_logits), _ptr(stream)),
                    "moe_lm_head_device")

    def sample(self, logits, temp: float, top_p: float, rng_state: int):
        """(tokens, next rng_state) for rows of logits, as sample_top_p."""
        lg = _f32(logits)
        lg = lg.reshape(-1, lg.shape[-1])
        st = C.c_uint32(rng_state)
        out = np.empty(lg.shape[0], np.int32)
        self._check(self.lib.moe_sample(self.ctx, _ptr(lg), lg.shape[0], lg.shape[1], temp, top_p, C.byref(st),
                                        _ptr(out)), "moe_sample")
        return out, st.value

    def sample_device(self, d_logits, n_tokens: int, vocab: int, temp: float, top_p: float, rng_state: int,
                      d_tokens, stream=None):
        self._check(self.lib.moe_sample_device(self.ctx, _ptr(d_logits), n_tokens, vocab, temp, top_p, rng_state,
                                               _ptr(d_tokens), _ptr(stream)), "moe_sample_device")

    # --------------------------------------------------------------- forward
    def forward(self, layer: int, h_post):
        """MoE block on host arrays: returns (out [T,H], idx [T,K], w [T,K])."""
        h = _f32(h_post).reshape(-1, self.cfg.hidden)
        T = h.shape[0]
        out = np.empty_like(h)
        idx = np.empty((T, self.cfg.top_k), np.int32)
        w = np.empty((T, self.cfg.top_k), np.float32)
        self._check(self.lib.moe_forward(self.ctx, layer, _ptr(h), T, _ptr(out), _ptr(idx), _ptr(w)), "moe_forward")
        return out, idx, w

    def forward_device(self, layer: int, d_h, n_tokens: int, d_out, d_idx=None, d_w=None, stream=None):
        self._check(self.lib.moe_forward_device(self.ctx, layer, _ptr(d_h), n_tokens, _ptr(d_out), _ptr(d_idx),
                                                _ptr(d_w), _ptr(stream)), "moe_forward_device")

    def check_error(self):
        """Waits for the context stream; raises MoeError if a kernel recorded
        an error (timed-out bounded wait, bad routing index) since the last
        check."""
        self._check(self.lib.moe_check_error(self.ctx), "moe_check_error")

    def experts_forward(self, layer: int, h_post, exp_idx, exp_w):
        """Routed experts with the routing given (metal_moe_forward)."""
        h = _f32(h_post).reshape(-1, self.cfg.hidden)
        T = h.shape[0]
        idx = np.ascontiguousarray(exp_idx, np.int32).reshape(T, -1)
        w = _f32(exp_w).reshape(T, -1)
        out = np.empty_like(h)
        self._check(self.lib.moe_experts_forward(self.ctx, layer, _ptr(h), T, _ptr(idx), _ptr(w), idx.shape[1],
                                                 _ptr(out)), "moe_experts_forward")
        return out

    def experts_forward_device(self, layer, d_h, n_tokens, d_idx, d_w, K, d_out, stream=None):
        self._check(self.lib.moe_experts_forward_device(self.ctx, layer, _ptr(d_h), n_tokens, _ptr(d_idx),
                                                        _ptr(d_w), K, _ptr(d_out), _ptr(stream)),
                    "moe_experts_forward_device")

    def shared_forward(self, layer: int, h_post):
        h = _f32(h_post).reshape(-1, self.cfg.hidden)
        out = np.empty_like(h)
        self._check(self.lib.moe_shared_forward(self.ctx, layer, _ptr(h), h.shape[0], _ptr(out)),
                    "moe_shared_forward")
        return out

    def route(self, logits, bias=None):
        lg = _f32(logits).reshape(-1, self.cfg.n_experts)
        T = lg.shape[0]
        b = None if bias is None else _f32(bias)
        idx = np.empty((T, self.cfg.top_k), np.int32)
        w = np.empty((T, self.cfg.top_k), np.float32)
        self._check(self.lib.moe_route(self.ctx, _ptr(lg), _ptr(b), T, _ptr(idx), _ptr(w)), "moe_route")
        return idx, w

    def prefill(self, layer: int, h_post):
        """Many tokens through one layer on the tensor-core path: (out, idx, w)."""
        h = _f32(h_post).reshape(-1, self.cfg.hidden)
        T = h.shape[0]
        out = np.empty_like(h)
        idx = np.empty((T, self.cfg.top_k), np.int32)
        w = np.empty((T, self.cfg.top_k), np.float32)
        self._check(self.lib.moe_prefill(self.ctx, layer, _ptr(h), T, _ptr(out), _ptr(idx), _ptr(w)), "moe_prefill")
        return out, idx, w

    def prefill_device(self, layer: int, d_h, n_tokens: int, d_out, d_idx=None, d_w=None, stream=None):
        self._check(self.lib.moe_prefill_device(self.ctx, layer, _ptr(d_h), n_tokens, _ptr(d_out), _ptr(d_idx),
                                                _ptr(d_w), _ptr(stream)), "moe_prefill_device")

    def forward_stack(self, first_layer: int, n_layers: int, hidden):
        h = _f32(hidden).reshape(-1, self.cfg.hidden).copy()
        self._check(self.lib.moe_forward_stack(self.ctx, first_layer, n_layers, _ptr(h), h.shape[0]),
                    "moe_forward_stack")
        return h

    def forward_stack_device(self, first_layer, n_layers, d_hidden, n_tokens, stream=None):
        self._check(self.lib.moe_forward_stack_device(self.ctx, first_layer, n_layers, _ptr(d_hidden), n_tokens,
                                                      _ptr(stream)), "moe_forward_stack_device")


def dequantize_row_q4_K(src, n: int) -> np.ndarray:
    """Device twin of quant.h:11."""
    s = np.ascontiguousarray(src, np.uint8)
    out = np.empty(n, np.float32)
    rc = load_library().moe_dequantize_row_q4_K(_ptr(s), _ptr(out), n)
    if rc != 0:
        raise MoeError(f"moe_dequantize_row_q4_K failed ({rc})")
    return out


def dequantize_row_q6_K(src, n: int) -> np.ndarray:
    """Device twin of quant.h:12."""
    s = np.ascontiguousarray(src, np.uint8)
    out = np.empty(n, np.float32)
    rc = load_library().moe_dequantize_row_q6_K(_ptr(s), _ptr(out), n)
    if rc != 0:
        raise MoeError(f"moe_dequantize_row_q6_K failed ({rc})")
    return out


__all__ = ["MoE", "MoeConfig", "MoeError", "TYPE_BF16", "TYPE_F16", "TYPE_F32", "TYPE_Q4_K", "TYPE_Q6_K", "dequantize_row_q4_K", "dequantize_row_q6_K",
           "get_unique_id", "load_library", "row_bytes"]
