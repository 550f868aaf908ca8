"""Plain-Python part of the layer's ABI: status codes, format codes, the
ctypes images of `MoEArgs` / `MoeDims` / the weight-file header, and
`LayerConfig` (one layer shape).

Nothing here loads libsparsemoe_b200.so, so this file can be loaded on its
own (by path) where the library must not be: the benchmark's reference arm
describes its workload with it and computes CAP with the CPU oracle instead.
The package binds CAP to the library's moe_capacity on import.
"""
from __future__ import annotations

import ctypes
import dataclasses

_capacity_fn = None


def set_capacity_fn(fn) -> None:
    """Binds the CAP function LayerConfig.capacity() uses:
    fn(tokens, top_k, num_experts, capacity_factor) -> int."""
    global _capacity_fn
    _capacity_fn = fn


MOE_OK = 0
MOE_ERR_INVALID_ARG = -1
MOE_ERR_UNSUPPORTED = -2
MOE_ERR_CUDA = -3
MOE_ERR_TIMEOUT = -4
MOE_ERR_NO_KERNEL = -5

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_INT8 = 2
DTYPE_FP8_BLOCK = 3
DTYPE_W4A16 = 4
DTYPE_INT8_CHANNEL = 5
DTYPE_NVFP4 = 6
DTYPE_INT4_PTX = 7   # the reference's capacity_int4_ptx format (packed-transposed per-tensor int4)
DTYPE_FP8 = 8        # the reference's capacity_fp8_ptx format (per-tensor e4m3)
ROUTER_SAME = 0
ROUTER_F32 = 1


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"moe error {code}: {msg}")
        self.code = code


_p = ctypes.c_void_p


class MoEArgs(ctypes.Structure):
    """ctypes image of `struct MoEArgs` (include/moe_args.h; reference include/moe_args.h:8-55)."""

    _fields_ = [
        ("input", _p), ("router_weights", _p),
        ("expert_up_proj_weights", _p), ("expert_gate_proj_weights", _p), ("expert_down_proj_weights", _p),
        ("expert_up_proj_weights_int8", _p), ("expert_gate_proj_weights_int8", _p),
        ("expert_down_proj_weights_int8", _p),
        ("expert_up_proj_weights_int4", _p), ("expert_gate_proj_weights_int4", _p),
        ("expert_down_proj_weights_int4", _p),
        ("expert_up_proj_weights_fp8", _p), ("expert_gate_proj_weights_fp8", _p),
        ("expert_down_proj_weights_fp8", _p),
        ("scale_up_w", ctypes.c_float), ("scale_gate_w", ctypes.c_float), ("scale_down_w", ctypes.c_float),
        ("scale_input_act", ctypes.c_float), ("scale_mid_act", ctypes.c_float),
        ("expert_logits", _p), ("selected_expert_indices", _p), ("selected_expert_weights", _p),
        ("expert_counts", _p), ("expert_token_ids", _p), ("expert_token_weights", _p),
        ("per_expert_wmma_inputs", _p), ("per_expert_wmma_inputs_int8", _p),
        ("per_expert_wmma_inputs_int4", _p), ("per_expert_wmma_inputs_fp8", _p),
        ("hidden_mlp_layer_1_out", _p), ("hidden_mlp_gate_out", _p), ("hidden_mlp_layer_1_out_fp16", _p),
        ("hidden_mlp_layer_1_out_int8", _p), ("hidden_mlp_layer_1_out_int4", _p),
        ("hidden_mlp_layer_1_out_fp8", _p), ("hidden_mlp_layer_2_out", _p),
        ("final_output", _p),
        ("num_batches", ctypes.c_int), ("use_capacity", ctypes.c_bool), ("cap", ctypes.c_int),
    ]


class MoeDims(ctypes.Structure):
    """ctypes image of `MoeDims` (include/sparsemoe_b200.h)."""

    _fields_ = [
        ("num_batches", ctypes.c_int), ("tokens", ctypes.c_int), ("d_model", ctypes.c_int),
        ("d_ff", ctypes.c_int), ("num_experts", ctypes.c_int), ("top_k", ctypes.c_int),
        ("capacity_factor", ctypes.c_float), ("cap", ctypes.c_int), ("dtype", ctypes.c_int),
        ("router_dtype", ctypes.c_int), ("router_bias", _p), ("output_16", _p),
        ("scratch", _p), ("scratch_bytes", ctypes.c_size_t),
        ("w_scale_gate", _p), ("w_scale_up", _p), ("w_scale_down", _p),
        ("w4_scale_gate", _p), ("w4_scale_up", _p), ("w4_scale_down", _p),
        ("w4_zero_gate", _p), ("w4_zero_up", _p), ("w4_zero_down", _p),
        ("fp4_global_gate", _p), ("fp4_global_up", _p), ("fp4_global_down", _p),
        ("slot_base", _p), ("act_scale", _p), ("skip_gather", ctypes.c_int),
        ("norm_weight", _p), ("norm_eps", ctypes.c_float), ("norm_out", _p), ("residual", _p),
    ]


class MoeWeightArray(ctypes.Structure):
    """ctypes image of `MoeWeightArray` (include/sparsemoe_b200.h)."""

    _fields_ = [("name", ctypes.c_char * 24), ("elem_bytes", ctypes.c_int32), ("kind", ctypes.c_int32),
                ("ndim", ctypes.c_int32), ("reserved", ctypes.c_int32), ("shape", ctypes.c_int64 * 4),
                ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


class MoeWeightFile(ctypes.Structure):
    """ctypes image of `MoeWeightFile` (include/sparsemoe_b200.h)."""

    _fields_ = [("magic", ctypes.c_char * 8), ("dtype", ctypes.c_int32), ("router_dtype", ctypes.c_int32),
                ("num_experts", ctypes.c_int32), ("d_model", ctypes.c_int32), ("d_ff", ctypes.c_int32),
                ("num_arrays", ctypes.c_int32), ("reserved", ctypes.c_int32), ("arrays", MoeWeightArray * 16)]


@dataclasses.dataclass(frozen=True)
class LayerConfig:
    """One layer shape.  `tokens` is per batch (routing and CAP are per batch)."""

    num_batches: int
    tokens: int
    d_model: int
    d_ff: int
    num_experts: int
    top_k: int
    capacity_factor: float
    dtype: int = DTYPE_F16
    router_f32: bool = False
    zipf_s: float = 0.0          # > 0: add a Zipf(s) popularity bias to the logits
    cap: int = 0                 # 0: computed; > 0: override; -1: no drop
    act_scale: float = 1.0       # per-tensor formats: s_in (the reference's placeholder is 1.0)
    mid_scale: float = 1.0       # per-tensor formats: s_mid

    @property
    def T(self) -> int:
        return self.num_batches * self.tokens

    @property
    def bf16(self) -> bool:
        return self.dtype == DTYPE_BF16

    @property
    def fp8(self) -> bool:
        return self.dtype == DTYPE_FP8_BLOCK

    @property
    def w4(self) -> bool:
        """4-bit packed weights (INT4 asymmetric g128 or NVFP4), bf16 activations."""
        return self.dtype in (DTYPE_W4A16, DTYPE_NVFP4)

    @property
    def nvfp4(self) -> bool:
        return self.dtype == DTYPE_NVFP4

    @property
    def act_bf16(self) -> bool:
        """Activations (x, router, 16-bit output) are bf16."""
        return self.dtype in (DTYPE_BF16, DTYPE_FP8_BLOCK, DTYPE_W4A16, DTYPE_INT8_CHANNEL, DTYPE_NVFP4)

    @property
    def int8(self) -> bool:
        """The reference's per-tensor int8 format."""
        return self.dtype == DTYPE_INT8

    @property
    def int8ch(self) -> bool:
        """int8 with per-output-channel weight scales and per-token activation scales."""
        return self.dtype == DTYPE_INT8_CHANNEL

    @property
    def int4ptx(self) -> bool:
        """The reference's int4 format: per-tensor int4 weights packed
        transposed ([E, N/2, K] bytes), int4 activations (one per byte)."""
        return self.dtype == DTYPE_INT4_PTX

    @property
    def fp8pt(self) -> bool:
        """The reference's fp8 format: per-tensor e4m3 weights and activations."""
        return self.dtype == DTYPE_FP8

    @property
    def per_tensor(self) -> bool:
        """A format with the reference's five per-tensor MoEArgs scales."""
        return self.dtype in (DTYPE_INT8, DTYPE_INT4_PTX, DTYPE_FP8)

    @property
    def channel_scaled(self) -> bool:
        """Weight scales travel in MoeDims.w_scale_* (FP8 blocks or int8 channels)."""
        return self.dtype in (DTYPE_FP8_BLOCK, DTYPE_INT8_CHANNEL)

    def capacity(self) -> int:
        if self.cap > 0:
            return self.cap
        if self.cap < 0:
            return self.tokens
        if _capacity_fn is None:
            raise RuntimeError("no CAP function bound (import sparsemoe_b200, or call set_capacity_fn)")
        return _capacity_fn(self.tokens, self.top_k, self.num_experts, self.capacity_factor)

    def dims(self, router_bias_ptr: int | None = None, out16_ptr: int | None = None,
             scratch_ptr: int | None = None, scratch_bytes: int = 0, w_scales=(None, None, None),
             w4=(None,) * 6, fp4_global=(None,) * 3) -> MoeDims:
        return MoeDims(self.num_batches, self.tokens, self.d_model, self.d_ff, self.num_experts, self.top_k,
                       self.capacity_factor, self.cap, self.dtype, ROUTER_F32 if self.router_f32 else ROUTER_SAME,
                       router_bias_ptr, out16_ptr, scratch_ptr, scratch_bytes, *w_scales, *w4, *fp4_global)
