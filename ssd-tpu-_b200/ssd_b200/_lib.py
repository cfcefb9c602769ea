"""ctypes binding of ``libssdverify.so`` (the sm_100a C ABI in include/ssd_verify.h).

The library is built in-tree (``make -C ssd-tpu-_b200/csrc``) next to this file.
There is no fallback: if the library is missing or a call fails, an exception
is raised.  Device buffers are torch tensors; streams are torch's current CUDA
stream unless one is passed.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libssdverify.so"

SSD_OK = 0
SSD_DTYPE_BF16 = 0
SSD_DTYPE_F32 = 1
SSD_ALIGN_REFERENCE = 0
SSD_ALIGN_STANDARD = 1
SSD_EPI_STORE, SSD_EPI_STORE_F32, SSD_EPI_RESIDUAL, SSD_EPI_GEGLU = 0, 1, 2, 3

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_u64 = C.c_uint64
_f = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes); mirrors include/ssd_verify.h
SIGNATURES = {
    "ssd_status_string": (C.c_char_p, [_i]),
    "ssd_abi_version": (_i, []),
    "ssd_verify_greedy_workspace_size": (_sz, [_i, _i, _i]),
    "ssd_verify_greedy": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _sz, _i, _i, _i]),
    "ssd_verify_greedy_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i]),
    "ssd_argmax_rows": (_i, [_p, _p, _i64, _i, _i, _p, _p, _sz]),
    "ssd_sample_rows": (_i, [_p, _p, _i64, _i, _i, _f, _u64, _u64, _p, _p, _sz]),
    "ssd_top_p_mask": (_i, [_p, _p, _i64, _i, _i, _f, _f]),
    "ssd_verify_sample_workspace_size": (_sz, [_i, _i, _i]),
    "ssd_verify_sample": (_i, [_p, _p, _p, _p, _p, _p, _f, _f, _f, _i, _p, _p, _p, _p, _sz, _i, _i, _i]),
    "ssd_uniform_fill": (_i, [_p, _p, _i64, _u64, _u64]),
    "ssd_page_allocate": (_i, [_p, _p, _p, _i, _p, _p, _p, _i, _p, _p, _p, _i, _i]),
    "ssd_page_rollback": (_i, [_p, _p, _p, _i, _p, _p, _p, _i, _p, _p, _p, _i, _i]),
    "ssd_page_free": (_i, [_p, _p, _p, _i, _p, _p, _i, _p, _p, _p, _i, _p, _i]),
    "ssd_page_fork": (_i, [_p, _p, _p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p, _i, _i, _i, _i]),
    "ssd_spec_cache_lookup": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _p, _i, _p, _p, _p, _p]),
    "ssd_kv_write": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p, _p, _p, _i, _i]),
    "ssd_paged_attention_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i]),
    "ssd_paged_verify_attention": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p, _p, _p, _f,
                                        _i, _i, _i, _i, _p, _sz]),
    "ssd_linear_workspace_size": (_sz, [_i, _i, _i]),
    "ssd_linear_max_m": (_i, []),
    "ssd_linear": (_i, [_p, _p, _p, _i, _p, _i, _i, _i, _i, _p, _sz]),
    "ssd_linear_rownorm": (_i, [_p, _p, _p, _i, _p, _i, _i, _i, _i, _f, _p, _sz]),
    "ssd_embed": (_i, [_p, _p, _p, _i, _p, _i, _i, _i]),
    "ssd_rmsnorm": (_i, [_p, _p, _p, _i, _p, _i, _i, _f]),
    "ssd_rope_kv_write": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p, _p, _p, _i,
                               _i, _i]),
    "ssd_gemma_scratch_size": (_sz, [_p, _i, _i, _i]),
    "ssd_gemma_forward": (_i, [_p, _p, _p]),
    "ssd_normal_fill": (_i, [_p, _p, _i, _i64, _f, _u64]),
    "ssd_comm_ctrl_bytes": (_sz, []),
    "ssd_comm_recv_bytes": (_sz, [_i, _i, _i]),
    "ssd_ipc_export": (_i, [_p, _p, C.POINTER(_sz)]),
    "ssd_ipc_import": (_i, [_p, _sz, C.POINTER(_p)]),
    "ssd_ipc_close": (_i, [_p, _sz]),
    "ssd_linear_allreduce": (_i, [_p, _p, _p, _p, _i, _i, _i, _p, _sz, _p]),
    "ssd_linear_allgather": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p, _sz, _p]),
}

SSD_MAX_TP = 8
SSD_ALLREDUCE_AUTO, SSD_ALLREDUCE_ALL_TO_ALL, SSD_ALLREDUCE_OWNER = 0, 1, 2


class CommC(C.Structure):
    """ssd_comm."""

    _fields_ = [
        ("rank", _i), ("world", _i), ("heaps", _p * SSD_MAX_TP), ("heap_bytes", _sz),
        ("ctrl_offset", _sz), ("recv_offset", _sz), ("recv_bytes", _sz), ("recv_rows", _i), ("recv_tiles", _i),
        ("allreduce_form", _i),
    ]


class GemmaWeightsC(C.Structure):
    """ssd_gemma_weights."""

    _fields_ = [
        ("num_layers", _i), ("d_model", _i), ("num_heads", _i), ("num_kv_heads", _i),
        ("head_dim", _i), ("ffn", _i), ("vocab", _i), ("eps", _f), ("dtype", _i),
        ("embed", _p), ("final_norm", _p),
        ("w_qkv", C.POINTER(_p)), ("w_o", C.POINTER(_p)), ("w_gate_up", C.POINTER(_p)), ("w_down", C.POINTER(_p)),
        ("rope_cos", _p), ("rope_sin", _p), ("rope_max_pos", _i),
        ("tp_rank", _i), ("tp_world", _i), ("qk_pairs", _i),
    ]


class GemmaBatchC(C.Structure):
    """ssd_gemma_batch."""

    _fields_ = [
        ("B", _i), ("T", _i), ("tokens", _p), ("seq_lens_before", _p), ("q_lens", _p),
        ("kv_pages", _p), ("num_blocks", _i), ("block_size", _i), ("block_tables", _p),
        ("max_blocks", _i), ("max_seq_len", _i), ("logits", _p), ("logits_last_only", _i),
        ("scratch", _p), ("scratch_bytes", _sz),
        ("prof_events", C.POINTER(_p)), ("prof_capacity", _i), ("prof_count", C.POINTER(_i)),
        ("prof_kind", C.POINTER(_i)),
        ("comm", C.POINTER(CommC)),
    ]


class SSDError(RuntimeError):
    pass


_LIB = None


def lib() -> C.CDLL:
    """Load the library once; raise if it is missing (no fallback path exists)."""
    global _LIB
    if _LIB is None:
        path = Path(os.environ.get("SSD_B200_LIB", LIB_PATH))
        if not path.exists():
            raise SSDError(
                f"{path} not found: build it with `make -C ssd-tpu-_b200/csrc` "
                "(the verify path has no CPU implementation)")
        so = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(so, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = so
    return _LIB


def check(rc: int, what: str) -> None:
    if rc != SSD_OK:
        msg = lib().ssd_status_string(rc).decode()
        raise SSDError(f"{what} failed: {msg} (status {rc})")


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def dtype_code(torch_dtype) -> int:
    import torch

    if torch_dtype == torch.bfloat16:
        return SSD_DTYPE_BF16
    if torch_dtype == torch.float32:
        return SSD_DTYPE_F32
    raise SSDError(f"unsupported dtype {torch_dtype}")
