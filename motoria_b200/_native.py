"""ctypes binding of libmiag.so (include/miag/miag.h).

The library is the product: a C ABI over hand-written sm_100a kernels.  This
module only declares its signatures.  It never substitutes anything for a
missing library -- import fails loudly instead.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmiag.so"


class Shape(C.Structure):
    """miag_shape (include/miag/miag.h)."""

    _fields_ = [
        ("dim", C.c_int32),
        ("n_layers", C.c_int32),
        ("n_experts", C.c_int32),
        ("n_active", C.c_int32),
        ("expert_hidden", C.c_int32),
        ("norm_topk", C.c_int32),
        ("norm_eps", C.c_float),
    ]


LOADER = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p)

# Every symbol include/miag/miag.h declares: name -> (restype, argtypes).
SIGNATURES = {
    "miag_blob_bytes": (C.c_size_t, [C.POINTER(Shape)]),
    "miag_open": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(Shape), C.c_int, C.c_char_p,
                            C.c_size_t]),
    "miag_close": (None, [C.c_void_p]),
    "miag_set_layer": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_char_p, C.c_size_t]),
    "miag_upload_experts": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                      C.c_size_t, C.c_char_p, C.c_size_t]),
    "miag_load_experts": (C.c_int, [C.c_void_p, LOADER, C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_upload_experts_device": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                             C.c_size_t, C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_moe": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_moe_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                 C.c_char_p, C.c_size_t]),
    "miag_moe_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                   C.c_char_p, C.c_size_t]),
    "miag_route_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                   C.c_size_t]),
    "miag_experts_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                     C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                     C.c_char_p, C.c_size_t]),
    "miag_combine_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_dx_stride": (C.c_int, [C.POINTER(Shape)]),
    "miag_ep_plan_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_char_p, C.c_size_t]),
    "miag_ep_pack_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                     C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                     C.c_size_t]),
    "miag_ep_buffer": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_char_p, C.c_size_t]),
    "miag_ep_open_peer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                    C.c_size_t]),
    "miag_ep_close_peers": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_experts_to_ranks_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                              C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                              C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint,
                                              C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_ep_wait_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_uint, C.c_void_p,
                                     C.c_char_p, C.c_size_t]),
    "miag_sync": (C.c_int, [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_selftest_wait_timeout": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_routing": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                               C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_router_logits": (C.c_int, [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_quantize_row_q8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "miag_matvec": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                              C.c_int, C.c_void_p]),
    "miag_last_launch_count": (C.c_int, [C.c_void_p]),
    "miag_set_prefill_kernel": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_set_transfer_chunks": (C.c_int, [C.c_void_p, C.c_int]),
    "miag_set_host_copy_threads": (C.c_int, [C.c_void_p, C.c_int]),
    "miag_prefill_kernel": (C.c_int, [C.c_void_p]),
    "miag_mia_write": (C.c_int, [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t]),
    "miag_mia_expert_blob_bytes": (C.c_size_t, [C.c_void_p]),
    "miag_nccl_unique_id": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_nccl_comm_init": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                      C.c_char_p, C.c_size_t]),
    "miag_nccl_comm_destroy": (None, [C.c_void_p]),
    "miag_ep_open": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_char_p,
                               C.c_size_t]),
    "miag_ep_close": (None, [C.c_void_p]),
    "miag_moe_ep_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                    C.c_char_p, C.c_size_t]),
    "miag_moe_ep": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_ep_rank": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                               C.c_void_p]),
    "miag_ep_last_received": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "miag_model_open": (C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_model_open_file": (C.c_int, [C.POINTER(C.c_void_p), C.c_char_p, C.c_int, C.c_int,
                                       C.c_char_p, C.c_size_t]),
    "miag_model_close": (None, [C.c_void_p]),
    "miag_model_synth": (C.c_int, [C.c_void_p, C.c_uint64, C.c_char_p, C.c_size_t]),
    "miag_model_step": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_model_step_async": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_model_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                      C.c_char_p, C.c_size_t]),
    "miag_model_generate_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                            C.c_char_p, C.c_size_t]),
    "miag_model_continue_async": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "miag_model_sync": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "miag_model_logits_device": (C.c_void_p, [C.c_void_p]),
    "miag_model_tokens_device": (C.c_void_p, [C.c_void_p]),
    "miag_model_stream": (C.c_void_p, [C.c_void_p]),
    "miag_model_moe": (C.c_void_p, [C.c_void_p]),
    "miag_model_launches_per_step": (C.c_int, [C.c_void_p]),
    "miag_model_uses_graph": (C.c_int, [C.c_void_p]),
    "miag_model_prefill_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_char_p,
                                           C.c_size_t]),
    "miag_model_prefill": (C.c_void_p, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_char_p,
                                         C.c_size_t]),
    "miag_model_set_batched_prefill": (C.c_int, [C.c_void_p, C.c_int]),
    "miag_model_set_sampler": (C.c_int, [C.c_void_p, C.c_float, C.c_float, C.c_uint64, C.c_char_p,
                                         C.c_size_t]),
    "miag_model_prefill_launches": (C.c_int, [C.c_void_p]),
    "miag_profile": (C.c_int, [C.c_void_p, C.c_int]),
    "miag_profile_stages": (C.c_int, []),
    "miag_profile_stage_name": (C.c_char_p, [C.c_int]),
    "miag_profile_read": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libmiag.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m motoria_b200.build` "
                "(libmiag has no CPU fallback)")
        dll = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(dll, name)
            fn.restype = res
            fn.argtypes = args
        _lib = dll
    return _lib


class MiagError(RuntimeError):
    pass


def check(rc: int, err: C.Array, what: str) -> None:
    if rc != 0:
        raise MiagError(f"{what}: {err.value.decode(errors='replace') or 'failed'}")


def errbuf() -> C.Array:
    return C.create_string_buffer(512)
