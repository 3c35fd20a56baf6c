"""ctypes binding of libstyx_moe.so (include/styx_moe.h, include/styx_residency.h,
include/styx_gguf.h, include/styx_attn.h).

There is no fallback: if the library is missing, importing the ops raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstyx_moe.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
HEADER = os.path.join(INCLUDE, "styx_moe.h")
HEADERS = [HEADER, os.path.join(INCLUDE, "styx_residency.h"), os.path.join(INCLUDE, "styx_gguf.h"),
           os.path.join(INCLUDE, "styx_attn.h")]

STYX_OK, STYX_EINVAL, STYX_ECUDA, STYX_ENOMEM, STYX_ETIMEOUT, STYX_EUNSUPPORTED = 0, -1, -2, -3, -4, -5
STYX_EIO, STYX_EEOF, STYX_EDATA = -6, -7, -8
F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
QTYPES = {"q8_0": Q8_0, "q4_K": Q4_K, "q5_K": Q5_K, "q6_K": Q6_K}
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
SKIP = 0xFFFFFFFF
IDS_PER_LAYER = 64
MEM_DEVICE, MEM_HOST = 0, 1
OPT_MOE_KERNELS, OPT_MOE_LAST_PATH, OPT_TRACE, OPT_MOE_LAYERS, OPT_EXCLUSIVE = 1, 2, 3, 4, 5
OPT_ATTN_KERNELS, OPT_ATTN_LAST_PATH, OPT_MOE_LAST_CLUSTER = 6, 7, 8
MOE_AUTO, MOE_FUSED, MOE_SPLIT, MOE_CLUSTER = 0, 1, 2, 3


class StyxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"styx error {code}: {msg}")
        self.code = code


class GgufTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("dims", C.POINTER(C.c_uint64)),
                ("ggml_type", C.c_uint32), ("offset", C.c_uint64), ("size_bytes", C.c_uint64)]


class ExpertTensor(C.Structure):
    _fields_ = [("full", C.c_void_p), ("hot", C.c_void_p), ("arena", C.c_void_p),
                ("slab_bytes", C.c_uint64), ("arena_slab_bytes", C.c_uint64),
                ("qtype", C.c_int32), ("n_hot", C.c_uint32), ("n_arena", C.c_uint32)]


class MoeLayer(C.Structure):
    _fields_ = [("ffn_norm", C.c_void_p), ("router", C.c_void_p), ("remap", C.c_void_p),
                ("pmap", C.c_void_p), ("gate", ExpertTensor), ("up", ExpertTensor),
                ("down", ExpertTensor)]


class RepinSwap(C.Structure):
    _fields_ = [("layer", C.c_int32), ("slot", C.c_int32), ("old_expert", C.c_uint32),
                ("new_expert", C.c_uint32)]


class MoeDims(C.Structure):
    _fields_ = [("n_embd", C.c_int32), ("n_ff", C.c_int32), ("n_expert", C.c_int32),
                ("n_expert_used", C.c_int32), ("norm_topk", C.c_int32), ("rms_eps", C.c_float)]


class DenseTensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("qtype", C.c_int32)]


class AttnDims(C.Structure):
    _fields_ = [("n_embd", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("qk_norm", C.c_int32), ("rms_eps", C.c_float), ("rope_base", C.c_float)]


class AttnLayer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("wq", DenseTensor), ("wk", DenseTensor), ("wv", DenseTensor),
                ("wo", DenseTensor), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)]


_vp, _i, _f, _u64 = C.c_void_p, C.c_int, C.c_float, C.c_uint64
_SIGS = {
    "styx_last_error": (C.c_char_p, []),
    "styx_init": (_i, [_i, C.POINTER(_vp)]),
    "styx_destroy": (None, [_vp]),
    "styx_vram_bytes": (_i, [_vp, C.POINTER(_u64)]),
    "styx_device_info": (_i, [_vp, C.POINTER(_i), C.c_char_p, _i]),
    "styx_check_device_error": (_i, [_vp, _vp]),
    "styx_set_option": (_i, [_vp, _i, C.c_int64]),
    "styx_get_option": (_i, [_vp, _i, C.POINTER(C.c_int64)]),
    "styx_alloc": (_i, [_vp, _u64, _i, C.POINTER(_vp)]),
    "styx_free": (_i, [_vp, _vp]),
    "styx_upload": (_i, [_vp, _vp, _u64, _vp, _u64, _vp]),
    "styx_download": (_i, [_vp, _vp, _vp, _u64, _u64, _vp]),
    "styx_copy": (_i, [_vp, _vp, _u64, _vp, _u64, _u64, _vp]),
    "styx_memset": (_i, [_vp, _vp, _i, _u64, _vp]),
    "styx_stream_create": (_i, [_vp, C.POINTER(_vp)]),
    "styx_stream_destroy": (_i, [_vp, _vp]),
    "styx_stream_sync": (_i, [_vp, _vp]),
    "styx_event_create": (_i, [_vp, C.POINTER(_vp)]),
    "styx_event_destroy": (_i, [_vp, _vp]),
    "styx_event_record": (_i, [_vp, _vp, _vp]),
    "styx_stream_wait_event": (_i, [_vp, _vp, _vp]),
    "styx_graph_begin": (_i, [_vp, _vp]),
    "styx_graph_end": (_i, [_vp, _vp, C.POINTER(_vp)]),
    "styx_graph_launch": (_i, [_vp, _vp, _vp]),
    "styx_graph_destroy": (_i, [_vp, _vp]),
    "styx_rms_norm": (_i, [_vp, _vp, _vp, _vp, _f, _i, _i, _vp]),
    "styx_matvec_f32": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "styx_topk_softmax": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "styx_mul_mat_vec_id": (_i, [_vp, _vp, _i, _vp, _u64, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp, _i]),
    "styx_swiglu": (_i, [_vp, _vp, _vp, _vp, _vp, _i]),
    "styx_moe_reduce": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i]),
    "styx_gather_slabs": (_i, [_vp, _vp, _vp, _vp, _vp, _u64, _u64, _u64, _vp, _vp, _vp,
                               _u64, _u64, _u64, _vp, _i, _i, _i]),
    "styx_gather_slabs_async": (_i, [_vp, _vp, _vp, _vp, _vp, _u64, _u64, _u64, _vp, _vp, _vp,
                                     _u64, _u64, _u64, _vp, _i, _i, _i]),
    "styx_moe_workspace_bytes": (_i, [C.POINTER(MoeDims), C.POINTER(_u64)]),
    "styx_moe_workspace_init": (_i, [_vp, _vp, _vp, _u64]),
    "styx_moe_workspace_view": (_i, [C.POINTER(MoeDims), _vp, _i, C.POINTER(_vp)]),
    "styx_moe_block": (_i, [_vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _vp, _vp,
                            _vp, _vp, _u64]),
    "styx_moe_block_noalloc": (_i, [_vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _vp, _vp, _vp]),
    "styx_moe_blocks": (_i, [_vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _i, _vp, _vp, _vp, _vp, _u64]),
    "styx_moe_block_ep": (_i, [_vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _vp, _vp, _vp, _vp,
                               _vp, _u64]),
    "styx_moe_combine": (_i, [_vp, _vp, _vp, _vp, _i, _i]),
    "styx_ep_open": (_i, [_vp, _i, _i, _i, _i, C.POINTER(_vp), _vp]),
    "styx_ep_connect": (_i, [_vp, _vp]),
    "styx_ep_combine": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "styx_ep_moe_block": (_i, [_vp, _vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _vp, _vp, _vp, _vp,
                               _u64]),
    "styx_ep_close": (_i, [_vp]),
    "styx_moe_batch_workspace_bytes": (_i, [C.POINTER(MoeDims), _i, C.POINTER(C.c_uint64)]),
    "styx_moe_block_batch": (_i, [_vp, _vp, C.POINTER(MoeDims), C.POINTER(MoeLayer), _i, _vp, _vp, _vp, _vp,
                                  C.c_uint64]),
    # include/styx_residency.h
    "styx_expert_budget": (_u64, [_u64, _u64, _u64, _u64, _u64, _i, _u64, _i]),
    "styx_arena_bytes": (_u64, [_i, _i, C.POINTER(_u64)]),
    "styx_residency_create": (_i, [_i, _i, _i, _u64, C.POINTER(_vp)]),
    "styx_residency_destroy": (None, [_vp]),
    "styx_residency_pin": (_i, [_vp, _vp, _vp, _vp, _i, _u64, C.POINTER(_i)]),
    "styx_residency_pin_csv": (_i, [_vp, C.c_char_p, C.c_size_t, _u64, C.POINTER(_i)]),
    "styx_residency_layer": (_i, [_vp, _i, _vp, _vp, C.POINTER(_i)]),
    "styx_residency_hits": (_i, [_vp, _i, _vp]),
    "styx_residency_maybe_repin": (_i, [_vp, _vp, _u64, _u64, _i, C.POINTER(RepinSwap), _i, C.POINTER(_i)]),
    "styx_residency_hot_cold": (_i, [_vp, _vp, _vp, _vp]),
    "styx_residency_prefetch_plan": (_i, [_vp, _vp, _vp, _vp]),
    # include/styx_gguf.h
    "styx_gguf_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
    "styx_gguf_open_memory": (_i, [_vp, _u64, C.POINTER(_vp)]),
    "styx_gguf_close": (None, [_vp]),
    "styx_gguf_version": (C.c_uint32, [_vp]),
    "styx_gguf_data_start": (_u64, [_vp]),
    "styx_gguf_file_bytes": (_u64, [_vp]),
    "styx_gguf_kv_count": (_u64, [_vp]),
    "styx_gguf_kv_key": (_i, [_vp, _u64, C.POINTER(C.c_char_p)]),
    "styx_gguf_kv_value": (_i, [_vp, _u64, C.POINTER(_u64)]),
    "styx_gguf_find_kv": (C.c_int64, [_vp, C.c_char_p]),
    "styx_gguf_node_type": (_i, [_vp, _u64, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(_u64)]),
    "styx_gguf_node_scalar": (_i, [_vp, _u64, _u64, _vp]),
    "styx_gguf_node_string": (_i, [_vp, _u64, _u64, C.POINTER(_vp), C.POINTER(_u64)]),
    "styx_gguf_node_elem": (_i, [_vp, _u64, _u64, C.POINTER(_u64)]),
    "styx_gguf_get_u32": (_i, [_vp, C.c_char_p, C.POINTER(C.c_uint32)]),
    "styx_gguf_get_f32": (_i, [_vp, C.c_char_p, C.POINTER(C.c_float)]),
    "styx_gguf_get_str": (_i, [_vp, C.c_char_p, C.POINTER(_vp), C.POINTER(_u64)]),
    "styx_gguf_tensor_count": (_u64, [_vp]),
    "styx_gguf_tensor": (_i, [_vp, _u64, C.POINTER(GgufTensorInfo)]),
    "styx_gguf_find_tensor": (C.c_int64, [_vp, C.c_char_p]),
    "styx_gguf_tensor_data": (_i, [_vp, _u64, C.POINTER(_vp)]),
    "styx_gguf_type_size": (_i, [C.c_uint32, C.POINTER(_u64), C.POINTER(_u64)]),
    "styx_gguf_tensor_bytes": (_i, [C.c_uint32, C.POINTER(_u64), C.c_uint32, C.POINTER(_u64)]),
    "styx_synth_quant": (_i, [_vp, _vp, _i, _vp, _u64, _i, _u64, _f]),
    "styx_synth_f32": (_i, [_vp, _vp, _vp, _u64, _u64, _u64, _f]),
    # include/styx_attn.h
    "styx_mul_mat_vec": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp, _vp]),
    "styx_mul_mat_vec_add": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp, _vp]),
    "styx_add_f32": (_i, [_vp, _vp, _vp, _vp, _vp, _i]),
    "styx_qk_norm_rope_kv": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _f, _vp, _vp, _vp, _i]),
    "styx_rope_neox": (_i, [_vp, _vp, _vp, _i, _i, _i, _f, _vp]),
    "styx_attn_workspace_bytes": (_i, [_i, _i, C.POINTER(_u64)]),
    "styx_attn_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp, _u64]),
    "styx_get_rows": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp, _i, _vp]),
    "styx_argmax_f32": (_i, [_vp, _vp, _vp, _i, _vp]),
    "styx_attn_block_workspace_bytes": (_i, [C.POINTER(AttnDims), C.POINTER(_u64)]),
    "styx_attn_block_workspace_init": (_i, [_vp, _vp, _vp, _u64]),
    "styx_attn_block": (_i, [_vp, _vp, C.POINTER(AttnDims), C.POINTER(AttnLayer), _vp, _i, _vp, _vp, _vp, _i,
                             _vp, _u64]),
}

_lib = None


def header_functions() -> list[str]:
    """Names of the functions the public headers (include/*.h) declare."""
    txt = "".join(open(h).read() for h in HEADERS)
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(styx_[a-z0-9_]+)\s*\(", txt)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m styx_b200.build` "
                "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != STYX_OK:
        msg = lib().styx_last_error()
        raise StyxError(rc, msg.decode() if msg else "")


def row_bytes(qtype: int, ncols: int) -> int:
    be, bb = BLOCK[qtype]
    assert ncols % be == 0
    return ncols // be * bb
