"""ctypes binding of ``librtr_b200.so`` (the C ABI declared in include/rtr_b200.h).

The library is loaded from the package directory only; a missing library or a
missing symbol raises immediately - there is no CPU fallback for any entry
point.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / 'librtr_b200.so'

RTR_OK, RTR_ERR_ARG, RTR_ERR_STATE, RTR_ERR_CUDA, RTR_ERR_DEVICE = range(5)
RTR_DTYPE_F32, RTR_DTYPE_BF16 = 0, 1
NUM_STEPS = 5

# Every symbol include/rtr_b200.h declares.
EXPORTS = (
    'rtr_session_create', 'rtr_session_destroy', 'rtr_last_error', 'rtr_set_stream',
    'rtr_load_weights', 'rtr_load_rope', 'rtr_load_constraints', 'rtr_prefill',
    'rtr_decode_step', 'rtr_read_results', 'rtr_generate', 'rtr_step_scores',
    'rtr_lookup_width', 'rtr_constraint_lookup', 'rtr_constraint_process',
    'rtr_synth_fill_host', 'rtr_synth_fill_device', 'rtr_launch', 'rtr_wait', 'rtr_get_report',
    'rtr_profile_gemms', 'rtr_constraint_process_static', 'rtr_gemm_check',
    'rtr_session_create_batched', 'rtr_launch_batch', 'rtr_wait_batch', 'rtr_generate_batch',
    'rtr_debug_wait_control', 'rtr_attention_check',
)


class ModelConfigC(ctypes.Structure):
    _fields_ = [('layers', ctypes.c_int32), ('hidden', ctypes.c_int32), ('heads', ctypes.c_int32),
                ('kv_heads', ctypes.c_int32), ('head_dim', ctypes.c_int32),
                ('intermediate', ctypes.c_int32), ('vocab', ctypes.c_int32),
                ('tied_embeddings', ctypes.c_int32), ('rms_eps', ctypes.c_float),
                ('rope_theta', ctypes.c_float), ('dtype', ctypes.c_int32),
                ('max_prefix', ctypes.c_int32), ('num_beams', ctypes.c_int32)]


class ConstraintTablesC(ctypes.Structure):
    _fields_ = [('offsets', ctypes.c_int32 * 3), ('sizes', ctypes.c_int32 * 3),
                ('table1', ctypes.POINTER(ctypes.c_int32)), ('width1', ctypes.c_int32),
                ('table2', ctypes.POINTER(ctypes.c_int32)), ('width2', ctypes.c_int32),
                ('valid', ctypes.POINTER(ctypes.c_uint8)),
                ('root', ctypes.c_int32 * 3),
                ('first_tokens', ctypes.POINTER(ctypes.c_int32)), ('n_first', ctypes.c_int32),
                ('newline', ctypes.c_int32), ('eos', ctypes.c_int32)]


class ResultC(ctypes.Structure):
    _fields_ = [('token_ids', ctypes.POINTER(ctypes.c_int32)),
                ('beam_indices', ctypes.POINTER(ctypes.c_int32)),
                ('sequence_logp', ctypes.POINTER(ctypes.c_float)),
                ('transition_logp', ctypes.POINTER(ctypes.c_float))]


class ReportC(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int64) for name in (
        'requests', 'kernel_launches', 'launches_per_request', 'graph_kernel_nodes', 'prefix_bytes_written',
        'prefix_bytes_reordered', 'suffix_bytes_written', 'suffix_bytes_gathered', 'weight_bytes',
        'device_bytes', 'h2d_bytes_per_request', 'd2h_bytes_per_request', 'tensor_core_gemm', 'norm_fold',
        'decode_attention', 'prefill_attention')]

    def as_dict(self):
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class NativeError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f'[rtr error {code}] {message}')
        self.code = code


_lib = None


def load():
    """Load the library (once); raises when it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f'{LIB_PATH.name} is not built; run `python -m rapidtinyrec_b200.build`')
    lib = ctypes.CDLL(str(LIB_PATH))
    missing = [name for name in EXPORTS if not hasattr(lib, name)]
    if missing:
        raise ImportError(f'{LIB_PATH.name} lacks symbols {missing}')
    P, I32, I64, F, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
    sig = {
        'rtr_session_create': (ctypes.POINTER(ModelConfigC), ctypes.c_int, ctypes.POINTER(P)),
        'rtr_session_destroy': (P,),
        'rtr_set_stream': (P, P),
        'rtr_load_weights': (P, ctypes.POINTER(P), I32, I32, I32),
        'rtr_load_rope': (P, P, P, I32),
        'rtr_load_constraints': (P, ctypes.POINTER(ConstraintTablesC)),
        'rtr_prefill': (P, P, I32, I32),
        'rtr_decode_step': (P, I32),
        'rtr_read_results': (P, ctypes.POINTER(ResultC)),
        'rtr_generate': (P, P, I32, ctypes.POINTER(ResultC)),
        'rtr_step_scores': (P, I32, P),
        'rtr_lookup_width': (P, I32, ctypes.POINTER(I32)),
        'rtr_constraint_lookup': (P, I32, P, I32, I32, P),
        'rtr_constraint_process': (P, I32, P, I32, I32, P, P),
        'rtr_synth_fill_host': (P, I64, U64, U64, F, F),
        'rtr_synth_fill_device': (P, I64, U64, U64, F, F, P),
        'rtr_launch': (P, P, I32, I32),
        'rtr_wait': (P, ctypes.POINTER(ResultC)),
        'rtr_get_report': (P, ctypes.POINTER(ReportC)),
        'rtr_profile_gemms': (P, I32, I32, ctypes.POINTER(F)),
        'rtr_gemm_check': (I32, P, P, P, I32, I32, I32, I32),
        'rtr_session_create_batched': (ctypes.POINTER(ModelConfigC), ctypes.c_int, I32, ctypes.POINTER(P)),
        'rtr_launch_batch': (P, P, P, I32, I32),
        'rtr_wait_batch': (P, ctypes.POINTER(ResultC)),
        'rtr_generate_batch': (P, P, P, I32, ctypes.POINTER(ResultC)),
        'rtr_constraint_process_static': (P, I32, P, I32, I32, P, P),
        'rtr_debug_wait_control': (I32, I64, I32),
        'rtr_attention_check': (I32, P, P, P, P, I32, I32, I32, I32, I32),
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = list(args)
        fn.restype = ctypes.c_int
    lib.rtr_last_error.argtypes = [P]
    lib.rtr_last_error.restype = ctypes.c_char_p
    _lib = lib
    return lib


def check(code, session=None):
    if code != RTR_OK:
        msg = load().rtr_last_error(session)
        raise NativeError(code, msg.decode() if msg else '')
    return code


def synth_fill(tensor, seed, tid, scale, offset):
    """Fill a contiguous float32 torch tensor with the synthetic stream (host or CUDA)."""
    import torch
    assert tensor.dtype == torch.float32 and tensor.is_contiguous()
    lib = load()
    if tensor.is_cuda:
        stream = torch.cuda.current_stream(tensor.device).cuda_stream
        with torch.cuda.device(tensor.device):
            check(lib.rtr_synth_fill_device(ctypes.c_void_p(tensor.data_ptr()), tensor.numel(), seed, tid,
                                            scale, offset, ctypes.c_void_p(stream)))
    else:
        check(lib.rtr_synth_fill_host(ctypes.c_void_p(tensor.data_ptr()), tensor.numel(), seed, tid,
                                      scale, offset))


def gemm(x, w, kernel=0):
    """``x @ w.T`` (fp32 CUDA tensors) through one of the engine's projection-GEMM
    kernels: 0 the engine's fp32 dispatch (the fp16-pair kernel), 1 the 64-row
    and 2 the 128-row tcgen05 3xTF32 kernels, 3 the bf16 kernel, 4 the FFMA
    kernel, 5 the tcgen05 fp16-pair kernel (``rtr_gemm_check``)."""
    import torch
    x = x.contiguous()
    w = w.contiguous()
    M, K = x.shape
    N = w.shape[0]
    c = torch.empty((M, N), dtype=torch.float32, device=x.device)
    torch.cuda.synchronize(x.device)
    check(load().rtr_gemm_check(x.device.index or 0, x.data_ptr(), w.data_ptr(), c.data_ptr(), M, N, K, kernel))
    return c


def attention(q, k, v, kernel):
    """Causal prefill attention of one layer through one kernel
    (``rtr_attention_check``): q [L, heads, D], k and v [kv_heads, L, D], fp32
    CUDA tensors; 0 FFMA, 1 tensor-core fp16 pairs, 2 bf16 FFMA, 3 bf16 tensor
    core."""
    import torch
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    L, heads, D = q.shape
    out = torch.empty_like(q)
    torch.cuda.synchronize(q.device)
    check(load().rtr_attention_check(q.device.index or 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                     L, heads, k.shape[0], D, kernel))
    return out


DEFAULT_WAIT_CYCLES = 2_000_000_000


def wait_control(device, wait_cycles=DEFAULT_WAIT_CYCLES, withhold_activation_copies=False):
    """Test control of the tensor-core GEMMs' bounded pipeline waits (``rtr_debug_wait_control``)."""
    check(load().rtr_debug_wait_control(device, int(wait_cycles), int(bool(withhold_activation_copies))))
