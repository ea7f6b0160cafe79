"""ctypes binding of the C ABI in include/mask_loss_b200.h.

The library is the in-tree ``mask_loss_b200/libmask_loss_b200.so`` built by
``mask_loss_b200.build``.  There is no fallback: if the library is missing or
does not load, importing an op raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmask_loss_b200.so")

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_f32 = ctypes.c_float
c_f64 = ctypes.c_double
c_vp = ctypes.c_void_p
c_sz = ctypes.c_size_t


class Dims(ctypes.Structure):
    _fields_ = [("L", c_i64), ("B", c_i64), ("Q", c_i64), ("H", c_i64), ("W", c_i64),
                ("Ht", c_i64), ("Wt", c_i64), ("C", c_i64), ("GT_total", c_i64)]


class Params(ctypes.Structure):
    _fields_ = [
        ("smooth", c_f32), ("sigmoid_scale", c_f32), ("dice_scale", c_f32), ("cls_scale", c_f32),
        ("background_index", c_i64),
        ("uncertainty_gamma", c_f32), ("uncertainty_gamma_min", c_f32),
        ("inf_thresh", c_f64), ("num_masks", c_f64),
        ("force_unmatched_class_to_background", c_i32), ("force_unmatched_masks_to_empty", c_i32),
        ("topk_matches", c_i64), ("strategy_id", c_i64),
        ("mask_gamma", c_f32), ("mask_alpha", c_f32), ("cls_gamma", c_f32), ("cls_alpha", c_f32),
        ("void_class_index", c_i64),
        ("use_softmax_label_loss", c_i32), ("normalize_uncertainty", c_i32),
        ("check_void_targets", c_i32), ("logits_dtype", c_i32),
    ]


# name -> (restype, argtypes); every function the header declares.
SIGNATURES = {
    "ml_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ml_last_error": (ctypes.c_char_p, []),
    "ml_version": (ctypes.c_int, []),
    "ml_gt_out": (c_i64, [c_i64, c_i64]),
    "ml_launch_count": (c_i64, []),
    "ml_profile_enable": (None, [ctypes.c_int]),
    "ml_profile_read": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int]),
    "ml_mask_matching_workspace_size": (c_sz, [ctypes.POINTER(Dims), ctypes.POINTER(Params)]),
    "ml_mask_matching_backward_workspace_size": (c_sz, [ctypes.POINTER(Dims), ctypes.POINTER(Params)]),
    "ml_match_workspace_size": (c_sz, [c_i64, c_i64, c_i64, c_i64]),
    "ml_pairwise_mask_loss_forward": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params),
                                                     c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp]),
    "ml_pairwise_mask_loss_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(Dims),
                                                             ctypes.POINTER(Params), c_vp, c_vp,
                                                             c_vp, c_vp, c_vp, c_vp]),
    "ml_noalloc_scratch_limit": (c_sz, []),
    "ml_cost_status": (ctypes.c_int, [ctypes.POINTER(c_i32)]),
    "ml_pairwise_label_loss_forward": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                                      c_f32, c_f32, c_f32, c_i32, c_vp, c_vp, c_vp,
                                                      c_vp]),
    "ml_match": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_f64, c_i64, c_i64, c_vp, c_vp,
                                c_vp, c_vp, c_sz, c_vp]),
    "ml_match_f64": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_f64, c_i64, c_i64, c_vp, c_vp,
                                    c_vp, c_vp]),
    "ml_mask_matching": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp,
                                        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                        c_sz, c_vp]),
    "ml_mask_matching_ex": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp,
                                           c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                           c_vp, c_sz, c_vp, c_vp]),
    "ml_mask_matching_ex2": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp,
                                            c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                            c_vp, c_vp, c_sz, c_vp, c_vp, c_vp]),
    "ml_count_masks": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp,
                                      c_vp, c_sz, c_vp]),
    "ml_dense_workspace_size": (c_sz, [ctypes.POINTER(Dims), ctypes.POINTER(Params)]),
    "ml_pairwise_mask_loss_dense_forward": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp, c_vp, c_vp, c_vp,
                                                           c_vp, c_sz, c_vp]),
    "ml_mask_matching_dense": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                              c_vp, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp]),
    "ml_mask_matching_dense_backward": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                       c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                       c_sz, c_vp]),
    "ml_semantic_workspace_size": (c_sz, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, ctypes.c_int32]),
    "ml_sigmoid_ce_forward": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_f32, c_f32, c_f32,
                                             c_f32, c_vp, c_vp, c_sz, c_vp]),
    "ml_sigmoid_ce_backward": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_f32, c_f32,
                                              c_f32, c_f32, c_vp, c_vp]),
    "ml_dice_forward": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_f32, c_f32, c_f32, c_vp, c_vp,
                                       c_vp, c_vp, c_vp, c_sz, c_vp]),
    "ml_dice_backward": (ctypes.c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_f32,
                                        c_f32, c_f32, c_vp, c_vp]),
    "ml_mask_matching_backward": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params),
                                                 c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                 c_vp, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp]),
    "ml_mask_matching_backward_ex": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params),
                                                    c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                    c_vp, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp, c_vp]),
    "ml_mask_matching_backward_ex2": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params),
                                                     c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                     c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_sz,
                                                     c_vp, c_vp, ctypes.c_int]),
    "ml_sampled_workspace_size": (c_sz, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_i64]),
    "ml_sampled_backward_workspace_size": (c_sz, [ctypes.POINTER(Dims), ctypes.POINTER(Params),
                                                  c_i64, c_i32]),
    "ml_pairwise_mask_loss_sampled_forward": (ctypes.c_int, [ctypes.POINTER(Dims),
                                                             ctypes.POINTER(Params), c_i64, c_i32,
                                                             c_i32, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                             c_vp, c_vp, c_sz, c_vp]),
    "ml_mask_matching_sampled": (ctypes.c_int, [ctypes.POINTER(Dims), ctypes.POINTER(Params), c_i64,
                                                c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_sz,
                                                c_vp]),
    "ml_mask_matching_sampled_backward": (ctypes.c_int, [ctypes.POINTER(Dims),
                                                         ctypes.POINTER(Params), c_i64, c_i32,
                                                         c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                         c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                         c_vp, c_vp, c_sz, c_vp]),
}

_LIB = None


def load() -> ctypes.CDLL:
    """Load the library (once).  Raises if it is missing: there is no fallback."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"mask_loss_b200: {LIB_PATH} is missing; build it with "
                "`python -m mask_loss_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def loaded() -> bool:
    return _LIB is not None


def check(rc: int) -> None:
    if rc != 0:
        lib = load()
        detail = lib.ml_last_error().decode()
        raise RuntimeError(detail or lib.ml_status_string(rc).decode())
