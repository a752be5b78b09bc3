"""ctypes binding of libptcg_b200.so (the C-ABI of include/ptcg_b200.h).

`lib()` loads the in-tree library and raises if it is missing -- there is no
CPU fallback for any computing entry point.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libptcg_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
HEADER = os.path.join(INCLUDE, "ptcg_b200.h")

P = C.c_void_p
F = C.c_float
I = C.c_int
L = C.c_long
FP = C.POINTER(C.c_float)


class PtcgShape(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "d", "heads", "ffn", "layers", "ltok", "nopt", "tok_f",
        "n_cards", "n_attacks", "n_skills")]

    @classmethod
    def from_shape(cls, s):
        return cls(s.d, s.heads, s.ffn, s.layers, s.ltok, s.nopt, s.tok_f,
                   s.n_cards, s.n_attacks, s.n_skills)


GRAD_HOOK = C.CFUNCTYPE(None, C.c_void_p, C.c_long, C.c_long, C.c_void_p)

_SIGS = {
    "ptcg_last_error": (C.c_char_p, []),
    "ptcg_abi_version": (I, []),
    "ptcg_obs_size": (L, [C.POINTER(PtcgShape)]),
    "ptcg_seat_column": (L, [C.POINTER(PtcgShape)]),
    "ptcg_obs_packed_bytes": (L, [C.POINTER(PtcgShape)]),
    "ptcg_obs_pack": (I, [C.POINTER(PtcgShape), P, L, P, C.POINTER(C.c_long)]),
    "ptcg_obs_unpack": (I, [C.POINTER(PtcgShape), P, L, P, P]),
    "ptcg_num_params": (I, [C.POINTER(PtcgShape)]),
    "ptcg_param_info": (I, [C.POINTER(PtcgShape), I, C.POINTER(C.c_char_p),
                            C.POINTER(C.c_long), C.POINTER(C.c_long)]),
    "ptcg_param_total": (L, [C.POINTER(PtcgShape)]),
    "ptcg_create": (I, [C.POINTER(PtcgShape), I, I, C.POINTER(P)]),
    "ptcg_destroy": (I, [P]),
    "ptcg_set_tables": (I, [P, P, P, P, P, P, P, P]),
    "ptcg_load_weights": (I, [P, P, L]),
    "ptcg_save_weights": (I, [P, P, L]),
    "ptcg_reserve": (I, [P, I, I]),
    "ptcg_save_weights_file": (I, [P, C.c_char_p]),
    "ptcg_load_weights_file": (I, [P, C.c_char_p]),
    "ptcg_save_state": (I, [P, C.c_char_p, L, L, I]),
    "ptcg_load_state": (I, [P, C.c_char_p, C.POINTER(C.c_long), C.POINTER(C.c_long)]),
    "ptcg_forward": (I, [P, P, I, P, P]),
    "ptcg_forward_train": (I, [P, P, I, P, P]),
    "ptcg_forward_sample": (I, [P, P, I, P, L, P, P, P, P, P, P]),
    "ptcg_backward": (I, [P, P, P, I, F, I, P]),
    "ptcg_workspace_create": (I, [P, I, C.POINTER(P)]),
    "ptcg_workspace_destroy": (I, [P]),
    "ptcg_forward_ws": (I, [P, P, P, I, P, P]),
    "ptcg_import_params": (I, [P, P, L, P]),
    "ptcg_ppo_loss": (I, [P, I, P, P, P, P, P, P, P, I, I, F, F, F, F,
                          P, P, P, P, P, P]),
    "ptcg_ppo_loss_noalloc": (I, [P, I, P, P, P, P, P, P, P, I, I, F, F, F, F,
                                  P, P, P, P, P]),
    "ptcg_adam_step": (I, [P, F, F, F, F, F, P, P, P]),
    "ptcg_sumsq": (I, [P, P, L, P, P]),
    "ptcg_adam_segments": (I, [P, P, P, I, P, F, F, F, F, F, P, P, P]),
    "ptcg_refresh_copies": (I, [P, P]),
    "ptcg_muon_step": (I, [P, F, F, F, F, F, P, P, P]),
    "ptcg_prio_replay": (I, [P, I, I, F, F, I, I, P, P, P, P, P, P]),
    "ptcg_select_copy": (I, [P, I, I, L, I, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
    "ptcg_index_copy": (I, [P, P, P, I, L, P]),
    "ptcg_sample_logits": (I, [P, I, I, P, L, P, P, P, P, P]),
    "ptcg_negamax_advantage": (I, [P, P, P, P, P, L, I, I, I, F, F, F, F, P, P]),
    "ptcg_set_grad_hook": (I, [P, GRAD_HOOK, P]),
    "ptcg_train_step": (I, [P, P, P, P, P, P, P, P, I, I, F, F, F, F, F, F, F,
                            F, F, I, P, P]),
    "ptcg_arena": (I, [P, I, C.POINTER(FP), C.POINTER(C.c_long)]),
    "ptcg_param_offset": (L, [P, I]),
    "ptcg_get_step": (I, [P, C.POINTER(C.c_long)]),
    "ptcg_set_step": (I, [P, L]),
    "ptcg_weights_checksum": (I, [P, P, P]),
    "ptcg_dp_unique_id": (I, [P]),
    "ptcg_dp_init": (I, [P, P, I, I]),
    "ptcg_dp_weights_agree": (I, [P, P, P]),
    "ptcg_dp_finalize": (I, [P, I]),
    "ptcg_kernel_timer": (I, [P, I]),
    "ptcg_launch_count": (C.c_longlong, []),
    "ptcg_kernel_timer_entries": (I, [P, I, P, P]),
    "ptcg_tensor_cores": (I, []),
    "ptcg_tc_profile": (I, [I, P]),
    "ptcg_eval_gelu": (I, [P, P, P, I, P]),
    "ptcg_attention_fwd": (I, [I, P, L, P, P, L, P, I, I, I, P]),
    "ptcg_attention_bwd": (I, [I, P, L, P, P, L, P, L, P, P, L, P, I, I, I, P]),
    "ptcg_device_error": (I, []),
    "ptcg_set_attention_impl": (I, [I]),
    "ptcg_get_attention_impl": (I, []),
    "ptcg_set_fused_mlp": (I, [I]),
    "ptcg_gemm": (I, [I, I, I, P, L, I, P, L, I, I, P, L, I, I, P]),
    "ptcg_gemm_ex": (I, [I, I, I, P, L, I, P, L, I, I, P, L, I, P, I, P, L, P, L, P, I, I, P]),
    "ptcg_kernel_timer_bytes": (I, [P, C.POINTER(C.c_double)]),
    "ptcg_kernel_timer_read": (I, [P, C.POINTER(C.c_double), C.POINTER(C.c_long),
                                   C.POINTER(C.c_double)]),
}

_lib = None


class PtcgError(RuntimeError):
    pass


def header_symbols():
    """Function names declared in the headers under include/ (the typedef'd
    function-pointer types of the plug-in header are not exports)."""
    names = set()
    for f in sorted(os.listdir(INCLUDE)):
        if not f.endswith(".h"):
            continue
        txt = open(os.path.join(INCLUDE, f)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        txt = re.sub(r"typedef[^;]*;", "", txt)
        names.update(re.findall(r"\b(ptcg_[a-z_0-9]+)\s*\(", txt))
    return sorted(names)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise PtcgError(f"{LIB_PATH} is missing: build it with "
                        "`python __graft_entry__.py build` (nvcc, sm_100a)")
    h = C.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(h, name)
        fn.restype = res
        fn.argtypes = args
    missing = [s for s in header_symbols() if not hasattr(h, s)]
    if missing:
        raise PtcgError(f"libptcg_b200.so lacks declared symbols: {missing}")
    _lib = h
    return h


def check(rc):
    if rc != 0:
        raise PtcgError(f"ptcg error {rc}: {lib().ptcg_last_error().decode()}")
    return rc


def obs_pack(shape, rows):
    """Observation rows (n, obs_size) float32 -> their compact transfer form,
    (n, ptcg_obs_packed_bytes) uint8 (ptcg_obs_pack, host only)."""
    import numpy as np
    h = lib()
    cs = PtcgShape.from_shape(shape)
    rows = np.ascontiguousarray(rows, np.float32)
    nb = h.ptcg_obs_packed_bytes(C.byref(cs))
    out = np.empty((rows.shape[0], nb), np.uint8)
    bad = C.c_long(-1)
    check(h.ptcg_obs_pack(C.byref(cs), rows.ctypes.data_as(P), rows.shape[0],
                          out.ctypes.data_as(P), C.byref(bad)))
    return out
