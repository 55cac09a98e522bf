"""bissimamba_b200 -- B200-native k-mamba scanND / convND hot path.

The product is the C-ABI shared library ``libkmamba_b200.so`` (declared in
``include/scan_nd.h`` and ``include/convnd.h``).  This module only binds it
with ctypes, mirroring the reference's C interface (``ScanNDParams``,
``scannd()``, ``om_scannd_forward/backward``, ``ConvNDParams``, ``convnd()``)
so Python callers and the tests use the same entry points a C caller links.

There is no CPU fallback: if the library is missing, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkmamba_b200.so")

_f = C.POINTER(C.c_float)
_l = C.POINTER(C.c_long)


class ScanNDParams(C.Structure):
    """Same field order and types as the reference include/scan_nd.h:40-69."""
    _fields_ = [
        ("max_ndims", C.c_long), ("max_state", C.c_long), ("use_fast_exp", C.c_int),
        ("dims", _l), ("ndims", C.c_long), ("D", C.c_long), ("M", C.c_long),
        ("x", C.c_void_p), ("A", C.c_void_p), ("B", C.c_void_p), ("C", C.c_void_p),
        ("delta", C.c_void_p), ("h", C.c_void_p), ("y", C.c_void_p),
        ("theta", C.c_void_p), ("lambda_", C.c_void_p),
        ("default_lambda", C.c_float), ("use_a_log_clamp", C.c_int), ("a_log_min", C.c_float),
        ("dA", C.c_void_p), ("dB", C.c_void_p), ("dC", C.c_void_p), ("ddelta", C.c_void_p),
        ("dlambda", C.c_void_p), ("dtheta", C.c_void_p),
    ]


class ConvNDParams(C.Structure):
    """Same layout as the reference include/convnd.h:10-23."""
    _fields_ = [
        ("input", C.c_void_p), ("kernel", C.c_void_p), ("bias", C.c_void_p),
        ("output", C.c_void_p), ("dy", C.c_void_p), ("dinput", C.c_void_p),
        ("dkernel", C.c_void_p), ("dbias", C.c_void_p), ("dims", _l),
        ("ndims", C.c_long), ("D", C.c_long), ("K", C.c_long),
    ]


class KMBlockScanParams(C.Structure):
    """include/kmamba_block.h"""
    _fields_ = [("ndims", C.c_long), ("dims", _l), ("L", C.c_long), ("N", C.c_long), ("R", C.c_long),
                ("u", C.c_void_p), ("dt", C.c_void_p), ("lambda_", C.c_void_p), ("B", C.c_void_p),
                ("C", C.c_void_p), ("A_log", C.c_void_p), ("theta", C.c_void_p),
                ("default_lambda", C.c_float), ("use_fast_exp", C.c_int),
                ("h", C.c_void_p), ("Bu", C.c_void_p), ("y", C.c_void_p), ("inputs_bf16", C.c_int)]


class KMBlockScanGrads(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("dB", "dC", "du", "ddt", "dlambda", "dA_log", "dtheta")]


class KMBlockConfig(C.Structure):
    _fields_ = [("dim", C.c_long), ("N", C.c_long), ("R", C.c_long), ("ndims", C.c_long), ("dims", _l),
                ("L", C.c_long), ("dt_min", C.c_float), ("dt_max", C.c_float), ("default_lambda", C.c_float),
                ("use_fast_exp", C.c_int), ("bf16_storage", C.c_int)]


BLOCK_FIELDS = ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "lambda_proj", "b_B", "b_C", "theta")


class KMBlockWeights(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in BLOCK_FIELDS]


class KMBlockGrads(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in BLOCK_FIELDS]


def block_config(dims, dim, N, R, dt_min=1e-3, dt_max=0.1, default_lambda=0.5, use_fast_exp=0, bf16=False):
    c = KMBlockConfig()
    darr = dims_array(dims)
    c._dims_keep = darr
    c.dim, c.N, c.R = int(dim), int(N), int(R)
    c.ndims = len(dims)
    c.dims = C.cast(darr, _l)
    L = 1
    for d in dims:
        L *= int(d)
    c.L = L
    c.dt_min, c.dt_max, c.default_lambda, c.use_fast_exp = dt_min, dt_max, default_lambda, use_fast_exp
    c.bf16_storage = int(bf16)
    return c


MAX_NDIMS = 32


class KMambaConfig(C.Structure):
    """Same layout as the reference include/kmamba.h:238-278."""
    _fields_ = [("max_ndims", C.c_long), ("max_state", C.c_long), ("use_fast_exp", C.c_int),
                ("vocab_size", C.c_size_t), ("dim", C.c_size_t), ("state_size", C.c_size_t),
                ("seq_len", C.c_size_t), ("n_layers", C.c_size_t), ("mimo_rank", C.c_size_t),
                ("dt_scale", C.c_float), ("dt_min", C.c_float), ("dt_max", C.c_float),
                ("default_lambda", C.c_float), ("use_a_log_clamp", C.c_int), ("a_log_min", C.c_float),
                ("spatial_ndims", C.c_long), ("spatial_dims", C.c_long * MAX_NDIMS),
                ("use_convnd", C.c_int), ("use_convnd_bias", C.c_int), ("convnd_K", C.c_long),
                ("convnd_ndims", C.c_long), ("pad_left", C.c_long * MAX_NDIMS), ("pad_right", C.c_long * MAX_NDIMS),
                ("d_conv", C.c_uint32), ("expand_factor", C.c_float), ("model_name", C.c_char * 64),
                ("vocab_data", C.c_void_p), ("gpu_device", C.c_int), ("weight_tying", C.c_int)]


class MBOptimConfig(C.Structure):
    _fields_ = [(k, C.c_float) for k in ("lr", "mu", "beta2", "eps", "clip_norm", "weight_decay")]


CONVND_FORWARD, CONVND_BACKWARD, CONVND_COMPLETE = 1, 2, 3

# every symbol the public headers declare (checked by the CPU tests)
EXPORTS = [
    "scannd_validate", "scannd", "scannd_ref_with_plan", "om_scannd_forward", "om_scannd_backward",
    "scannd_batched", "scannd_backward_batched", "scannd_forward_async", "scannd_backward_async",
    "scannd_backward_ex", "kmb_last_backward_path",
    "convnd_kernel_volume", "convnd_forward_wavefront", "convnd_backward_wavefront", "convnd",
    "om_convnd_forward", "om_convnd_backward", "convnd_status", "convnd_batched_async",
    "convnd_backward_noalloc", "convnd_backward_noalloc_error",
    "wavefront_nd_validate_dims", "wavefront_nd_total_points", "wavefront_nd_max_level",
    "wavefront_nd_row_major_offset", "wavefront_nd_level_size", "wavefront_nd_for_level",
    "wavefront_nd_for_each_level", "km_wavefront_plan_create", "km_wavefront_plan_free",
    "km_wavefront_plan_matches_dims", "km_wavefront_plan_level_size", "km_wavefront_plan_level_offsets",
    "km_wavefront_plan_iter_forward", "km_wavefront_plan_iter_reverse",
    "kmb_last_error", "kmb_clear_error", "kmb_device_status", "kmb_last_forward_path", "kmb_set_force_generic",
    "kmb_set_scan_exp2", "kmb_get_scan_exp2", "kmb_init_tensor", "kmb_set_sm_reserve",
    "kmamba_distributed_split_batch", "kmamba_distributed_split_layers", "kmamba_distributed_init_nccl",
    "kmamba_distributed_fini_nccl", "kmamba_allreduce_gradients_nccl", "kmamba_broadcast_params_nccl",
    "kmb_dist_unique_id", "kmb_dist_init", "kmb_dist_exchange_id", "kmb_dist_world_size", "kmb_dist_rank",
    "kmb_dist_allreduce_async", "kmb_dist_allgather_async", "kmb_dist_broadcast_async", "kmb_dist_scannd_backward",
    "kmb_dist_convnd_backward", "kmb_dist_model_train_step",
    "kser_writer_create", "kser_writer_add_vocab", "kser_writer_add_tensor", "kser_writer_finalize", "kser_writer_free",
    "kser_reader_open", "kser_reader_config", "kser_reader_is_valid", "kser_reader_load_vocab", "kser_reader_load_tensor",
    "kser_reader_count_tensors", "kser_reader_get_tensor_info", "kser_reader_close", "kser_file_info", "kser_quantize",
    "kser_dequantize", "kser_dtype_size", "kser_sha256", "kmamba_save_ser", "kmamba_load_ser", "kmb_load_ser_ex",
    "kmamba_ser_info", "kmamba_save_checkpoint_ser", "kmamba_load_checkpoint_ser",
    "kmb_blockscan_forward", "kmb_blockscan_set_strips", "kmb_blockscan_last_forward_path", "kmb_blockscan_set_backward_strips",
    "kmb_blockscan_last_backward_path", "kmb_blockscan_backward", "kmb_blockscan_backward_ex", "kmb_block_activation_floats",
    "kmb_block_forward", "kmb_block_backward", "kmb_block_set_tensor_cores", "kmb_block_last_projection_path", "kmb_block_last_dx_path", "cuda_block_forward", "cuda_block_backward",
    "kmamba_config_set_defaults", "kmamba_optim_config_set_defaults", "kmamba_create", "kmamba_free",
    "kmamba_init", "kmamba_enable_training", "kmamba_forward", "kmamba_train_batch", "kmamba_train_step",
    "kmamba_get_config", "kmamba_step_count", "kmamba_update_lr", "kmamba_get_tensor", "kmamba_set_tensor",
    "kmb_model_forward_backward", "kmb_model_optimizer_step", "kmb_model_grad_arena", "kmb_model_param_arena", "kmb_model_tensor_offset",
    "kmb_gemm_f32", "kmb_gemm_bf16", "kmb_gemm_set_f32_kind", "kmb_gemm_get_f32_kind", "kmb_gemm_set_f32_flush", "kmb_gemm_last_path",
]

_lib = None


def lib():
    """Load libkmamba_b200.so (build it first with ``bissimamba_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m bissimamba_b200.build` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        P = C.POINTER(ScanNDParams)
        Q = C.POINTER(ConvNDParams)
        for n in ("scannd_validate", "scannd", "om_scannd_forward", "om_scannd_backward"):
            getattr(L, n).argtypes = [P]
            getattr(L, n).restype = C.c_int
        L.scannd_batched.argtypes = [P, C.c_long]
        L.scannd_backward_batched.argtypes = [P, C.c_long, C.c_void_p]
        L.scannd_forward_async.argtypes = [P, C.c_long, C.c_void_p]
        L.scannd_backward_async.argtypes = [P, C.c_long, C.c_void_p, C.c_void_p]
        L.scannd_backward_ex.argtypes = [P, C.c_long, C.c_void_p, C.c_int, C.c_void_p]
        L.scannd_ref_with_plan.argtypes = [P, C.c_void_p]
        L.convnd.argtypes = [Q, C.c_int]
        L.convnd.restype = None
        L.convnd_batched_async.argtypes = [Q, C.c_long, C.c_int, C.c_void_p]
        L.om_convnd_forward.argtypes = [Q]
        L.convnd_backward_noalloc.argtypes = [Q, C.c_long, C.c_void_p]
        L.convnd_backward_noalloc_error.restype = C.c_char_p
        L.om_convnd_backward.argtypes = [Q]
        L.convnd_forward_wavefront.argtypes = [Q, C.c_void_p]
        L.convnd_forward_wavefront.restype = None
        L.convnd_backward_wavefront.argtypes = [Q, C.c_void_p]
        L.convnd_backward_wavefront.restype = None
        L.convnd_kernel_volume.argtypes = [C.c_long, C.c_long]
        L.convnd_kernel_volume.restype = C.c_long
        L.kmb_last_error.restype = C.c_char_p
        KC = C.POINTER(KMambaConfig)
        L.kmamba_config_set_defaults.argtypes = [KC]
        L.kmamba_config_set_defaults.restype = None
        L.kmamba_optim_config_set_defaults.argtypes = [C.POINTER(MBOptimConfig)]
        L.kmamba_optim_config_set_defaults.restype = None
        L.kmamba_create.argtypes = [KC]
        L.kmamba_create.restype = C.c_void_p
        L.kmamba_free.argtypes = [C.c_void_p]
        L.kmamba_free.restype = None
        L.kmamba_init.argtypes = [C.c_void_p, C.c_uint32]
        L.kmb_init_tensor.argtypes = [C.c_void_p, C.c_uint32, C.c_char_p, C.c_void_p, C.c_long]
        L.kmb_init_tensor.restype = C.c_long
        vp, sz = C.c_void_p, C.c_size_t
        L.kmamba_distributed_split_batch.argtypes = [vp, sz, sz]
        L.kmamba_distributed_split_batch.restype = None
        L.kmamba_distributed_split_layers.argtypes = [vp, sz, sz]
        L.kmamba_distributed_split_layers.restype = None
        L.kmamba_distributed_init_nccl.argtypes = [C.c_int, C.c_int]
        L.kmamba_distributed_init_nccl.restype = vp
        L.kmamba_distributed_fini_nccl.argtypes = [vp]
        L.kmamba_distributed_fini_nccl.restype = None
        L.kmamba_allreduce_gradients_nccl.argtypes = [vp, vp, sz]
        L.kmamba_broadcast_params_nccl.argtypes = [vp, vp, sz]
        L.kmb_dist_unique_id.argtypes = [vp]
        L.kmb_dist_init.argtypes = [vp, C.c_int, C.c_int, C.c_int]
        L.kmb_dist_init.restype = vp
        L.kmb_dist_exchange_id.argtypes = [vp, C.c_int, C.c_int, C.c_char_p, C.c_int]
        L.kmb_dist_world_size.argtypes = [vp]
        L.kmb_dist_rank.argtypes = [vp]
        L.kmb_dist_allreduce_async.argtypes = [vp, vp, sz, C.c_float, vp]
        L.kmb_dist_allgather_async.argtypes = [vp, vp, vp, sz, vp]
        L.kmb_dist_broadcast_async.argtypes = [vp, vp, sz, C.c_int, vp]
        L.kmb_dist_scannd_backward.argtypes = [vp, vp, C.c_long, vp, C.c_int, vp]
        L.kmb_dist_convnd_backward.argtypes = [vp, vp, C.c_long, vp]
        L.kmb_dist_model_train_step.argtypes = [vp, vp, vp, sz, sz, vp]
        L.kmb_dist_model_train_step.restype = C.c_float
        for fn in ("kser_writer_create", "kser_reader_open", "kser_reader_config", "kser_reader_load_tensor",
                   "kser_reader_get_tensor_info", "kmamba_load_ser", "kmb_load_ser_ex"):
            getattr(L, fn).restype = vp
        L.kser_writer_create.argtypes = [C.c_char_p, vp]
        L.kser_writer_add_vocab.argtypes = [vp, C.c_uint32, C.c_char_p, C.c_uint16]
        L.kser_writer_add_tensor.argtypes = [vp, C.c_char_p, vp, vp, C.c_int, C.c_int]
        L.kser_writer_finalize.argtypes = [vp]
        L.kser_writer_free.argtypes = [vp]
        L.kser_writer_free.restype = None
        L.kser_reader_open.argtypes = [C.c_char_p]
        L.kser_reader_config.argtypes = [vp]
        L.kser_reader_is_valid.argtypes = [vp]
        L.kser_reader_load_tensor.argtypes = [vp, C.c_char_p]
        L.kser_reader_count_tensors.argtypes = [vp]
        L.kser_reader_count_tensors.restype = C.c_uint64
        L.kser_reader_get_tensor_info.argtypes = [vp, C.c_uint64]
        L.kser_reader_close.argtypes = [vp]
        L.kser_reader_close.restype = None
        L.kser_quantize.argtypes = [vp, vp, C.c_uint64, C.c_int]
        L.kser_dequantize.argtypes = [vp, vp, C.c_uint64, C.c_int]
        L.kser_sha256.argtypes = [vp, sz, vp]
        L.kser_sha256.restype = None
        L.kmamba_save_ser.argtypes = [vp, C.c_char_p, C.c_int]
        L.kmamba_load_ser.argtypes = [C.c_char_p, C.c_int]
        L.kmb_load_ser_ex.argtypes = [C.c_char_p, C.c_int, vp]
        L.kmamba_enable_training.argtypes = [C.c_void_p, C.POINTER(MBOptimConfig), C.c_float, C.c_float]
        L.kmamba_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.kmamba_train_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        L.kmamba_train_batch.restype = C.c_float
        L.kmamba_train_step.argtypes = [C.c_void_p, C.c_void_p]
        L.kmamba_train_step.restype = C.c_float
        L.kmamba_get_tensor.argtypes = [C.c_void_p, C.c_char_p]
        L.kmamba_get_tensor.restype = _f
        L.kmamba_set_tensor.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p]
        L.kmamba_step_count.argtypes = [C.c_void_p]
        L.kmamba_step_count.restype = C.c_size_t
        L.kmamba_update_lr.argtypes = [C.c_void_p, C.c_float, C.c_float]
        L.kmamba_update_lr.restype = None
        ll = C.c_longlong
        L.kmb_gemm_f32.argtypes = [C.c_int, C.c_int, ll, ll, ll, vp, ll, vp, ll, vp, ll, C.c_int, vp]
        L.kmb_gemm_bf16.argtypes = [C.c_int, ll, ll, ll, vp, ll, vp, ll, vp, ll, C.c_int, vp]
        L.kmb_gemm_set_f32_kind.argtypes = [C.c_int]
        L.kmb_gemm_set_f32_flush.argtypes = [C.c_int]
        L.kmamba_get_config.argtypes = [C.c_void_p]
        L.kmamba_get_config.restype = KC
        L.kmb_model_forward_backward.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
        L.kmb_model_forward_backward.restype = C.c_float
        L.kmb_model_optimizer_step.argtypes = [C.c_void_p, C.c_void_p]
        L.kmb_model_grad_arena.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
        L.kmb_model_grad_arena.restype = C.c_void_p
        L.kmb_model_tensor_offset.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        L.kmb_model_param_arena.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
        L.kmb_model_param_arena.restype = C.c_void_p
        L.kmb_block_activation_floats.argtypes = [C.POINTER(KMBlockConfig), C.c_long]
        L.kmb_block_activation_floats.restype = C.c_size_t
        L.kmb_block_forward.argtypes = [C.POINTER(KMBlockConfig), C.POINTER(KMBlockWeights), C.c_void_p,
                                        C.c_void_p, C.c_long, C.c_void_p, C.c_void_p]
        L.kmb_block_backward.argtypes = [C.POINTER(KMBlockConfig), C.POINTER(KMBlockWeights), C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.POINTER(KMBlockGrads), C.c_long, C.c_void_p,
                                         C.c_void_p]
        L.kmb_blockscan_forward.argtypes = [C.POINTER(KMBlockScanParams), C.c_long, C.c_void_p]
        L.kmb_blockscan_backward.argtypes = [C.POINTER(KMBlockScanParams), C.c_long, C.c_void_p,
                                             C.POINTER(KMBlockScanGrads), C.c_void_p]
        L.kmb_blockscan_backward_ex.argtypes = [C.POINTER(KMBlockScanParams), C.c_long, C.c_void_p,
                                                C.POINTER(KMBlockScanGrads), C.c_int, C.c_void_p]
        L.kmb_blockscan_set_backward_strips.argtypes = [C.c_int]
        L.kmb_blockscan_set_backward_strips.restype = None
        L.kmb_set_force_generic.argtypes = [C.c_int]
        L.kmb_set_force_generic.restype = None
        L.kmb_set_scan_exp2.argtypes = [C.c_int]
        L.kmb_set_scan_exp2.restype = None
        L.kmb_set_sm_reserve.argtypes = [C.c_int]
        L.kmb_set_sm_reserve.restype = None
        L.km_wavefront_plan_create.argtypes = [_l, C.c_long, C.c_long]
        L.km_wavefront_plan_create.restype = C.c_void_p
        L.km_wavefront_plan_free.argtypes = [C.c_void_p]
        L.km_wavefront_plan_level_size.argtypes = [C.c_void_p, C.c_long]
        L.km_wavefront_plan_level_size.restype = C.c_long
        L.km_wavefront_plan_level_offsets.argtypes = [C.c_void_p, C.c_long]
        L.km_wavefront_plan_level_offsets.restype = _l
        L.wavefront_nd_level_size.argtypes = [_l, C.c_long, C.c_long]
        L.wavefront_nd_level_size.restype = C.c_long
        L.wavefront_nd_total_points.argtypes = [_l, C.c_long]
        L.wavefront_nd_total_points.restype = C.c_long
        L.wavefront_nd_max_level.argtypes = [_l, C.c_long]
        L.wavefront_nd_max_level.restype = C.c_long
        _lib = L
    return _lib


def last_error() -> str:
    return lib().kmb_last_error().decode()


def _ptr(t):
    """Data pointer of a tensor / numpy array / None."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


def dims_array(dims):
    arr = (C.c_long * len(dims))(*[int(d) for d in dims])
    return arr


def scan_params(dims, D, M, x, A, B, Cm, delta, h, y, theta=None, lam=None, default_lambda=0.5,
                use_fast_exp=0, use_a_log_clamp=0, a_log_min=-1e-5, grads=None):
    """Build a ScanNDParams (single-item layout; batched calls use the same
    struct with contiguous [batch, ...] buffers).  Keeps the dims array alive
    on the returned object."""
    p = ScanNDParams()
    darr = dims_array(dims)
    p._dims_keep = darr
    p.max_ndims = 32
    p.max_state = 0
    p.use_fast_exp = int(use_fast_exp)
    p.dims = C.cast(darr, _l)
    p.ndims = len(dims)
    p.D, p.M = int(D), int(M)
    p.x, p.A, p.B, p.C, p.delta = _ptr(x), _ptr(A), _ptr(B), _ptr(Cm), _ptr(delta)
    p.h, p.y = _ptr(h), _ptr(y)
    p.theta, p.lambda_ = _ptr(theta), _ptr(lam)
    p.default_lambda = float(default_lambda)
    p.use_a_log_clamp = int(use_a_log_clamp)
    p.a_log_min = float(a_log_min)
    g = grads or {}
    for k in ("dA", "dB", "dC", "ddelta", "dlambda", "dtheta"):
        setattr(p, k, _ptr(g.get(k)))
    return p


def conv_params(dims, D, K, inp=None, kernel=None, bias=None, out=None, dy=None, dinput=None,
                dkernel=None, dbias=None):
    p = ConvNDParams()
    darr = dims_array(dims)
    p._dims_keep = darr
    p.input, p.kernel, p.bias, p.output = _ptr(inp), _ptr(kernel), _ptr(bias), _ptr(out)
    p.dy, p.dinput, p.dkernel, p.dbias = _ptr(dy), _ptr(dinput), _ptr(dkernel), _ptr(dbias)
    p.dims = C.cast(darr, _l)
    p.ndims = len(dims)
    p.D, p.K = int(D), int(K)
    return p


def check(rc: int, what: str = "call"):
    if rc != 0:
        raise RuntimeError(f"{what} failed: {last_error()}")


def blockscan_params(dims, N, R, u, dt, lam, B, Cm, A_log, theta, h, Bu, y, default_lambda=0.5, use_fast_exp=0):
    p = KMBlockScanParams()
    darr = dims_array(dims)
    p._dims_keep = darr
    p.ndims = len(dims)
    p.dims = C.cast(darr, _l)
    L = 1
    for d in dims:
        L *= int(d)
    p.L, p.N, p.R = L, int(N), int(R)
    p.u, p.dt, p.lambda_, p.B, p.C = _ptr(u), _ptr(dt), _ptr(lam), _ptr(B), _ptr(Cm)
    p.A_log, p.theta = _ptr(A_log), _ptr(theta)
    p.default_lambda = float(default_lambda)
    p.use_fast_exp = int(use_fast_exp)
    p.h, p.Bu, p.y = _ptr(h), _ptr(Bu), _ptr(y)
    return p


def model_config(dims, vocab, dim, N, R, n_layers):
    """KMambaConfig with the reference defaults and the given shape."""
    c = KMambaConfig()
    lib().kmamba_config_set_defaults(C.byref(c))
    L = 1
    for d in dims:
        L *= int(d)
    c.vocab_size, c.dim, c.state_size, c.seq_len = vocab, dim, N, L
    c.n_layers, c.mimo_rank = n_layers, R
    c.spatial_ndims = len(dims)
    for i, d in enumerate(dims):
        c.spatial_dims[i] = int(d)
    return c


class DeviceArray:
    """Minimal __cuda_array_interface__ view of a library-owned device buffer
    (float32), so torch.as_tensor can read it without copying."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3}
