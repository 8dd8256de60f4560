"""ctypes binding of libember_b200.so (the C-ABI declared in include/ember.h,
include/ember_ops.h and include/ember_cuda.h).

The prototypes for the public API are the ones emberllm's own Python bindings
declare (bindings/python/emberllm.py:89-109); the rest cover the op-level
entry points and this library's extensions. Loading the library needs no GPU;
calling into the token loop without a usable sm_100 device ends the process
through the library's fatal-error convention, so callers check
``cuda_available()`` first.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libember_b200.so")

_P = ctypes.c_void_p
_FP = ctypes.POINTER(ctypes.c_float)
_IP = ctypes.POINTER(ctypes.c_int)


class EmberHeader(ctypes.Structure):
    """Layout of the 256-byte .ember header (ref src/ember.h:53-83)."""

    _pack_ = 1
    _fields_ = [
        ("magic", ctypes.c_char * 4), ("version", ctypes.c_uint32),
        ("header_bytes", ctypes.c_uint64),
        ("dim", ctypes.c_int32), ("hidden_dim", ctypes.c_int32), ("n_layers", ctypes.c_int32),
        ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32), ("max_seq_len", ctypes.c_int32),
        ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
        ("flags", ctypes.c_uint32), ("rope_style", ctypes.c_int32),
        ("bos_token_id", ctypes.c_int32), ("eos_token_id", ctypes.c_int32),
        ("eos_token_id2", ctypes.c_int32), ("n_tensors", ctypes.c_int32),
        ("tokenizer_type", ctypes.c_int32), ("default_top_k", ctypes.c_int32),
        ("default_temp", ctypes.c_float), ("default_top_p", ctypes.c_float),
        ("tokenizer_offset", ctypes.c_uint64), ("tokenizer_size", ctypes.c_uint64),
        ("tensor_table_offset", ctypes.c_uint64), ("tensor_table_size", ctypes.c_uint64),
        ("reserved", ctypes.c_uint8 * 128),
    ]


assert ctypes.sizeof(EmberHeader) == 256


class EmberSampleParams(ctypes.Structure):
    """The sampler settings of ember_sample_device (include/ember_cuda.h)."""

    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("min_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float),
                ("presence_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float)]

# every symbol the headers declare, grouped by header (tests check the exports)
PUBLIC_SYMBOLS = [
    "ember_model_load", "ember_model_free", "ember_model_header", "ember_model_tensor",
    "ember_model_data", "ember_state_new", "ember_state_new_ex", "ember_state_free",
    "ember_forward", "ember_prefill", "ember_quantize_file",
]
OPS_SYMBOLS = [
    "ember_f16_to_f32", "ember_f32_to_f16", "ember_quantize_q8_0", "ember_quantize_q4_0",
    "ember_matmul", "ember_matmul_batch", "ember_threads_init", "ember_threads_shutdown",
    "ember_nthreads", "ember_parallel_for", "ember_should_parallel", "ember_die",
    "ember_xmalloc", "ember_xcalloc", "ember_xrealloc",
]
CUDA_SYMBOLS = [
    "ember_cuda_model_upload", "ember_cuda_model_free", "ember_cuda_model_bytes",
    "ember_cuda_state_new", "ember_cuda_state_free", "ember_cuda_forward", "ember_cuda_prefill",
    "ember_cuda_greedy", "ember_cuda_state_host_logits", "ember_cuda_state_stream",
    "ember_cuda_state_logits_dev", "ember_cuda_state_launches_per_step", "ember_cuda_state_launches_per_token", "ember_cuda_state_persistent",
    "ember_cuda_error",
    "ember_cuda_available", "ember_cuda_profile_step", "ember_cuda_mark", "ember_cuda_elapsed_ms",
    "ember_cuda_time_kernel", "ember_cuda_argmax_static", "ember_host_expf_params",
    "ember_host_expf_emulated",
    "ember_host_rope_table", "ember_forward_greedy", "ember_state_cuda", "ember_cuda_sample",
    "ember_sample_device",
    "ember_cuda_batch_new", "ember_cuda_batch_free", "ember_cuda_batch_prefill", "ember_cuda_batch_greedy",
    "ember_cuda_batch_stream", "ember_batch_new", "ember_batch_cuda", "ember_batch_free", "ember_batch_prefill",
    "ember_batch_greedy",
]

_lib = None


def load(path=None):
    """Load (once) and return the library with its prototypes set."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("EMBER_B200_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `make -C emberllm_b200` "
            "(or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    lib.ember_model_load.restype = _P
    lib.ember_model_load.argtypes = [ctypes.c_char_p]
    lib.ember_model_free.argtypes = [_P]
    lib.ember_model_header.restype = ctypes.POINTER(EmberHeader)
    lib.ember_model_header.argtypes = [_P]
    lib.ember_model_tensor.restype = _P
    lib.ember_model_tensor.argtypes = [_P, ctypes.c_char_p]
    lib.ember_model_data.restype = _P
    lib.ember_model_data.argtypes = [_P, _P]
    lib.ember_state_new.restype = _P
    lib.ember_state_new.argtypes = [_P, ctypes.c_int]
    lib.ember_state_new_ex.restype = _P
    lib.ember_state_new_ex.argtypes = [_P, ctypes.c_int, ctypes.c_int]
    lib.ember_state_free.argtypes = [_P]
    lib.ember_forward.restype = _FP
    lib.ember_forward.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
    lib.ember_prefill.restype = _FP
    lib.ember_prefill.argtypes = [_P, _P, _IP, ctypes.c_int, ctypes.c_int]
    lib.ember_quantize_file.restype = ctypes.c_int
    lib.ember_quantize_file.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.ember_f16_to_f32.restype = ctypes.c_float
    lib.ember_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.ember_f32_to_f16.restype = ctypes.c_uint16
    lib.ember_f32_to_f16.argtypes = [ctypes.c_float]
    lib.ember_quantize_q8_0.argtypes = [_P, _P, ctypes.c_int]
    lib.ember_quantize_q4_0.argtypes = [_P, _P, ctypes.c_int]
    lib.ember_matmul.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
    lib.ember_matmul_batch.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, _P]
    lib.ember_threads_init.argtypes = [ctypes.c_int]
    lib.ember_nthreads.restype = ctypes.c_int
    lib.ember_forward_greedy.restype = _FP
    lib.ember_forward_greedy.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _IP]
    lib.ember_state_cuda.restype = _P
    lib.ember_state_cuda.argtypes = [_P]
    lib.ember_batch_new.restype = _P
    lib.ember_batch_new.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.ember_batch_free.argtypes = [_P]
    lib.ember_batch_prefill.restype = _FP
    lib.ember_batch_prefill.argtypes = [_P, ctypes.c_int, _IP, ctypes.c_int]
    lib.ember_batch_greedy.argtypes = [_P, _IP, _IP, ctypes.c_int, _IP, _FP]
    lib.ember_cuda_batch_stream.restype = _P
    lib.ember_cuda_batch_stream.argtypes = [_P]
    lib.ember_batch_cuda.restype = _P
    lib.ember_batch_cuda.argtypes = [_P]
    lib.ember_cuda_state_stream.restype = _P
    lib.ember_cuda_state_stream.argtypes = [_P]
    lib.ember_cuda_state_logits_dev.restype = _P
    lib.ember_cuda_state_logits_dev.argtypes = [_P]
    lib.ember_cuda_state_launches_per_step.restype = ctypes.c_int
    lib.ember_cuda_state_launches_per_step.argtypes = [_P]
    lib.ember_cuda_state_launches_per_token.restype = ctypes.c_int
    lib.ember_cuda_state_launches_per_token.argtypes = [_P]
    lib.ember_cuda_state_persistent.restype = ctypes.c_int
    lib.ember_cuda_state_persistent.argtypes = [_P, ctypes.POINTER(ctypes.c_char_p)]
    lib.ember_cuda_sample.restype = ctypes.c_int
    lib.ember_cuda_sample.argtypes = [_P, ctypes.POINTER(EmberSampleParams), ctypes.c_float, _IP, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_int)]
    lib.ember_sample_device.restype = ctypes.c_int
    lib.ember_sample_device.argtypes = [_P, ctypes.POINTER(EmberSampleParams), ctypes.POINTER(ctypes.c_uint64),
                                        _IP, ctypes.c_int]
    lib.ember_cuda_greedy.restype = ctypes.c_int
    lib.ember_cuda_greedy.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _IP, _FP]
    lib.ember_cuda_error.restype = ctypes.c_char_p
    lib.ember_cuda_available.restype = ctypes.c_int
    lib.ember_cuda_model_bytes.restype = ctypes.c_uint64
    lib.ember_cuda_model_bytes.argtypes = [_P]
    lib.ember_host_rope_table.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    _lib = lib
    return lib


def cuda_available():
    """True when the library loads and sees an sm_100-class device."""
    try:
        return bool(load().ember_cuda_available())
    except OSError:
        return False
