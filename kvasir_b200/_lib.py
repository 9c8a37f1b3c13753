"""ctypes binding of libkvasir_b200.so (the C ABI declared in include/kvasir_b200.h).

The library is loaded from kvasir_b200/_lib/ (built in-tree by
kvasir_b200/build.py).  There is no fallback: if the library is missing or
fails to load, importing the ops raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libkvasir_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "kvasir_b200.h")

(KVB_OK, KVB_ERR_SHAPE, KVB_ERR_CUDA, KVB_ERR_UNSUPPORTED, KVB_ERR_DEVICE, KVB_ERR_CONFIG,
 KVB_ERR_IO) = range(7)
KVB_BF16, KVB_F16 = 0, 1
KVB_CKPT_BF16, KVB_CKPT_F16, KVB_CKPT_F32, KVB_CKPT_OTHER = range(4)
KVB_NOALLOC_SCRATCH_BYTES = 8 << 20  # include/kvasir_b200.h

_sz = C.c_size_t
_p = C.c_void_p
_i32p = C.POINTER(C.c_int32)
_f32p = C.POINTER(C.c_float)
_int = C.c_int


class DecoderConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_layers", C.c_int32),
                ("n_q", C.c_int32), ("n_kv", C.c_int32), ("head_dim", C.c_int32),
                ("vocab", C.c_int32), ("max_seq", C.c_int32), ("n_seq", C.c_int32),
                ("eps", C.c_float), ("dtype", C.c_int32)]


class DecoderWeights(C.Structure):
    _fields_ = [("embed", _p), ("final_norm", _p), ("attn_norm", C.POINTER(_p)),
                ("w_qkv", C.POINTER(_p)), ("w_o", C.POINTER(_p)), ("mlp_norm", C.POINTER(_p)),
                ("w_gu", C.POINTER(_p)), ("w_down", C.POINTER(_p))]


# name -> (restype, argtypes)
SIGNATURES = {
    "kvb_last_error": (C.c_char_p, []),
    "kvb_version": (C.c_char_p, []),
    "kvb_device_error": (_int, [C.POINTER(C.c_uint32)]),
    "kvb_embedding_gather": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _int]),
    "kvb_rmsnorm": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, C.c_float, _int]),
    "kvb_embedding_rmsnorm": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _sz,
                                     C.c_float, _int]),
    "kvb_rope_inplace": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _sz, _sz, _int]),
    "kvb_silu_mul": (_int, [_p, _p, _sz, _p, _sz, _sz, _sz, _int]),
    "kvb_add_inplace": (_int, [_p, _p, _sz, _p, _sz, _int]),
    "kvb_bf16_to_f16": (_int, [_p, _p, _sz, _p, _sz, _p, _sz]),
    "kvb_kv_append": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _int]),
    "kvb_attention": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _sz, _sz, _sz,
                             _p, _sz, _int]),
    "kvb_attention_workspace_bytes": (_sz, [_sz, _sz, _sz, _sz, _sz]),
    "kvb_blas_create": (_int, [C.POINTER(_p)]),
    "kvb_blas_destroy": (_int, [_p]),
    "kvb_blas_set_workspace": (_int, [_p, _p, _sz]),
    "kvb_blas_set_autotune": (_int, [_p, _int]),
    "kvb_linear": (_int, [_p, _p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _int, _int]),
    "kvb_rope_table": (_int, [_sz, C.c_double, _int, C.c_double, C.c_double, C.c_double,
                              C.c_double, _sz, _p, _p]),
    "kvb_rope_kv_append": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _p, _sz, _sz, _sz, _sz, _sz, _sz,
                                  _sz, _int]),
    "kvb_rope_kv_append_batched": (_int, [_p, _p, _sz, _p, _p, _p, _sz, _p, _p, _sz, _sz, _sz,
                                          _sz, _sz, _sz, _int]),
    "kvb_rope_kv_append_prefill": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _p, _sz, _sz, _sz, _sz,
                                          _sz, _sz, _sz, _sz, _int]),
    "kvb_rope_kv_append_paged": (_int, [_p, _p, _sz, _sz, _p, _p, _p, _sz, _p, _p, _sz, _p, _sz,
                                        _sz, _sz, _sz, _sz, _int]),
    "kvb_attention_prefill_paged": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _sz, _sz, _p, _sz, _sz,
                                           _sz, _sz, _sz, _sz, _sz, _int]),
    "kvb_attention_decode_paged": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _sz, _sz, _p, _sz, _sz,
                                          _sz, _sz, _sz, C.c_float, _p, _sz, _p, _sz, _int]),
    "kvb_add_rmsnorm": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, C.c_float, _int]),
    "kvb_attention_decode": (_int, [_p, _p, _sz, _p, _p, _sz, _sz, _p, _sz, _sz, _sz, _sz, _sz,
                                    _sz, C.c_float, _p, _sz, _p, _sz, _int]),
    "kvb_attention_decode_workspace_bytes": (_sz, [_sz, _sz, _sz, _sz, _sz]),
    "kvb_attention_decode_noalloc": (_int, [_p, _p, _sz, _p, _p, _sz, _sz, _p, _sz, _sz, _sz, _sz,
                                            _sz, _sz, C.c_float, _p, _sz, _int]),
    "kvb_attention_prefill": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _sz, _sz, _sz, _sz, _sz, _sz,
                                     _sz, _sz, _int]),
    "kvb_attention_prefill_f32": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _sz, _sz, _sz, _sz, _sz, _sz,
                                     _sz, _sz, _int]),
    "kvb_argmax_f32": (_int, [_p, _p, _sz, _sz, _p, _p, _p]),
    "kvb_lm_head_argmax_workspace_bytes": (_sz, [_sz]),
    "kvb_decoder_set_fused_lm_head": (_int, [_p, _int]),
    "kvb_lm_head_argmax": (_int, [_p, _p, _sz, _p, _sz, _sz, _sz, _sz, _p, _sz, _p, _p, _p, _int]),
    "kvb_linear_rows": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _int, _int]),
    "kvb_linear_silu_mul": (_int, [_p, _p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _int, _int]),
    "kvb_decoder_set_row_projections": (_int, [_p, _int]),
    "kvb_rope_attention_decode_paged": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _p, _sz, _p, _sz, _sz,
                                               _p, _sz, _sz, _sz, _sz, _sz, C.c_float, _p, _sz, _p,
                                               _sz, _int]),
    "kvb_rope_attention_decode": (_int, [_p, _p, _sz, _p, _p, _sz, _p, _p, _sz, _sz, _p, _sz, _sz,
                                         _sz, _sz, _sz, _sz, C.c_float, _p, _sz, _p, _sz, _int]),
    "kvb_decoder_workspace_bytes": (_sz, [C.POINTER(DecoderConfig)]),
    "kvb_decoder_create": (_int, [C.POINTER(_p), C.POINTER(DecoderConfig),
                                  C.POINTER(DecoderWeights), _p, _p, _p, _p, _p, _sz]),
    "kvb_decoder_destroy": (_int, [_p]),
    "kvb_decoder_use_paged_cache": (_int, [_p, _p, _p, _sz, _p, _sz, _sz]),
    "kvb_decoder_set_lengths": (_int, [_p, _p, _p]),
    "kvb_decoder_ids_in": (_p, [_p]),
    "kvb_decoder_ids_out": (_p, [_p]),
    "kvb_decoder_logits": (_p, [_p]),
    "kvb_decoder_step": (_int, [_p, _p]),
    "kvb_decoder_step_host": (_int, [_p, _p, _p, _p]),
    "kvb_decoder_launches_per_step": (_int, [_p, C.POINTER(_int), C.POINTER(_int)]),
    "kvb_decoder_set_lm_head": (_int, [_p, _p]),
    "kvb_decoder_set_sampling": (_int, [_p, C.c_float, C.c_float, C.c_uint64]),
    "kvb_sample_f32": (_int, [_p, _p, _sz, _sz, C.c_float, C.c_float, C.c_uint64, _p, _p, _p, _p]),
    "kvb_checkpoint_open": (_int, [C.POINTER(_p), C.c_char_p]),
    "kvb_checkpoint_close": (_int, [_p]),
    "kvb_checkpoint_num_tensors": (_sz, [_p]),
    "kvb_checkpoint_tensor": (_int, [_p, C.c_char_p, C.POINTER(_int), C.POINTER(_int),
                                     C.POINTER(C.c_uint64)]),
    "kvb_checkpoint_load_rows": (_int, [_p, _p, C.POINTER(C.c_char_p), C.POINTER(C.c_uint64), _sz,
                                        C.c_uint64, _p, _sz, _int, _p]),
    "kvb_selftest_wait_timeout": (_int, [_p, C.c_uint32]),
}


def header_symbols(path: str = HEADER) -> list[str]:
    """Function names declared in include/kvasir_b200.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvb_[a-z0-9_]+)\s*\(", text)))


_lib = None


def lib() -> C.CDLL:
    """Load the library (once).  Raises OSError if it is missing: build it with
    `python -m kvasir_b200.build`."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing; build it with `python -m kvasir_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib
