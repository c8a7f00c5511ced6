"""ctypes binding of libfastmd_b200.so (the C ABI declared in include/fastmd_b200.h).

This is the only route from Python to the kernels. A missing or unloadable
library raises ``FastMDLibraryError``: there is no CPU fallback anywhere in
the package.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().with_name("libfastmd_b200.so")


class FastMDLibraryError(RuntimeError):
    """libfastmd_b200.so is missing, failed to load, or a call returned an error status."""


class FmdCatPart(ctypes.Structure):
    _fields_ = [("src", c_void_p), ("index", c_void_p), ("ld", c_int64), ("n_src", c_int64),
                ("width", c_int32), ("_pad", c_int32)]


class FmdGemmProblem(ctypes.Structure):
    """One problem of fmd_gemm_tf32x3_grouped (the arguments of fmd_gemm_tf32x3)."""
    _fields_ = [("x", c_void_p), ("ldx", c_int64), ("w_hi", c_void_p), ("w_lo", c_void_p), ("ldw", c_int64),
                ("bias", c_void_p), ("c", c_void_p), ("ldc", c_int64), ("y", c_void_p), ("ldy", c_int64),
                ("m", c_int64), ("n", c_int32), ("k", c_int32), ("act", c_int32), ("accumulate", c_int32)]


_P = c_void_p  # every device pointer and the stream travel as void*
_I64, _I32 = c_int64, c_int32

# name -> argument types (restype is int32 fmd_status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "fmd_version": [],
    "fmd_status_string": [_I32],
    "fmd_last_error": [],
    "fmd_gather_cat": [POINTER(FmdCatPart), _I32, _I64, _P, _I64, _P, _P],
    "fmd_aligned_gather_cat3": [_P, _I64, _P, _I64, _I64, _P, _P, _I64, _I32, _P, _P, _P],
    "fmd_gather_rows_bwd": [_P, _I64, _I32, _I32, _P, _P, _I64, _P, _I64, _I32, _P],
    "fmd_gather_rows_bwd_long": [_P, _I64, _I32, _I32, _P, _P, _I64, _P, _I64, _I32, _P],
    "fmd_copy_rows": [_P, _I64, _P, _I64, _I64, _I32, _P],
    "fmd_csr_offsets_sorted": [_P, _I64, _I64, _P, _P],
    "fmd_csr_build_workspace_bytes": [_I64, _I64, POINTER(c_size_t)],
    "fmd_csr_build": [_P, _I64, _I64, _P, _P, _P, c_size_t, _P, _P],
    "fmd_csr_segment_sum": [_P, _I64, _P, _I64, _P, _P, _I64, _I32, _I64, _P, _I64, _P],
    "fmd_csr_segment_sum_bwd": [_P, _P, _I64, _P, _I64, _P, _I64, _I64, _I32, _I64, _P, _P, _P, _P],
    "fmd_cell_list_workspace_bytes": [_P, c_float, _I64, _I32, POINTER(c_size_t)],
    "fmd_candidates_build": [_P, _P, _I64, _I32, c_float, _I32, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P],
    "fmd_refilter_workspace_bytes": [_I64, _I32, POINTER(c_size_t)],
    "fmd_refilter_edges": [_P, _P, _I64, _I32, _P, _P, _P, _P, _P, _I32, c_float, c_float, _I64, _P, _I32, _P, _P,
                           _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P],
    "fmd_refilter_edges_noalloc": [_P, _P, _I64, _I32, _P, _P, _P, _P, _P, _I32, c_float, c_float, _I64, _P, _I32,
                                   _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "fmd_neighbor_list_workspace_bytes": [_P, c_float, _I64, _I32, POINTER(c_size_t)],
    "fmd_neighbor_list": [_P, _P, _I64, c_float, _I32, _I64, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P],
    "fmd_gemm_f32": [_P, _I64, _P, _I64, _P, _I64, _I32, _P, _P, _I64, _P, _I64, _I64, _I32, _I32, _I32, _I32, _P],
    "fmd_gated_ln": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, c_float, c_float, _P, _P, _P, _P, _P, _P],
    "fmd_gated_ln_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P],
    "fmd_column_sum_workspace_bytes": [_I64, _I32, POINTER(c_size_t)],
    "fmd_column_sum": [_P, _I64, _I32, _I64, _P, c_size_t, _P, _P],
    "fmd_pair_aggregate": [_I32, _P, _I64, _P, _I64, _I32, _P, _P, _P],
    "fmd_residual_add": [_I32, _P, _I64, _P, _I64, _P, _I64, _I32, _P, _I64, _P],
    "fmd_reverse_pairs_workspace_bytes": [_I64, POINTER(c_size_t)],
    "fmd_reverse_pairs": [_P, _P, _P, _I64, _I64, _I32, _P, c_size_t, _P, _P, _P, _P, _P],
    "fmd_line_graph_workspace_bytes": [_I64, _I64, POINTER(c_size_t)],
    "fmd_line_graph": [_P, _P, _P, _I64, _I64, c_float, _I32, _I64, _P, c_size_t, _P, _P, _P, _P],
    "fmd_model_positions_f64": [_P, _I64, _P, _P, _P, _P],
    "fmd_pad_vector_override": [_P, _I64, _P, _P, _P],
    "fmd_bond_graph_workspace_bytes": [_I64, _I64, POINTER(c_size_t)],
    "fmd_bond_graph": [_P, _P, _I64, _P, _P, _P, _I64, _I64, c_float, _I32, _I64, _P, _P, c_size_t, _P, _P, _P, _P,
                       _P, _P],
    "fmd_gather_add_silu": [_P, _I64, POINTER(FmdCatPart), _I32, _P, _I64, _I32, _P, _P, _P, _P, _P],
    "fmd_silu_pair_bwd": [_P, _P, _P, _I64, _I32, _P, _I64, _P],
    "fmd_segment_attention": [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I32, _I64, _P, _P, _P, _P, _P, _P],
    "fmd_segment_attention_bwd": [_P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I64, _P, _I64, _P,
                                  _I64, _P, _P],
    "fmd_paired_segment_attention_bwd_rows": [_P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                              _P, _P, _I64, _I64, _I32, _I64, _P, _I64, _P, _I64, _P, _P, _P],
    "fmd_tf32_mma_rate": [_I32, _P, _P],
    "fmd_wait_probe": [_I32, _P, _P],
    "fmd_tf32_split": [_P, _I64, _I64, _I64, _I32, _P, _P, _I64, _P],
    "fmd_gemm_tf32x3": [_P, _I64, _P, _P, _I64, _P, _P, _I64, _P, _I64, _I64, _I32, _I32, _I32, _I32, _P, _P],
    "fmd_gemm_tf32x3_grouped": [POINTER(FmdGemmProblem), _I32, _P, _P],
    "fmd_matris_geometry": [_P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P],
    "fmd_matris_bessel": [_P, _P, _I64, _I64, _P, _P, _I32, c_float, c_float, c_float, _P, _P, _I64, _P],
    "fmd_matris_bessel_bwd": [_P, _P, _I64, _I64, _P, _P, _I32, c_float, c_float, c_float, _P, _P, _I64, _P, _P],
    "fmd_matris_threebody": [_P, _P, _I64, _I64, _P, _I32, _P, _I64, _P, _P],
    "fmd_matris_threebody_bwd": [_P, _P, _I64, _I64, _P, _I32, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _P],
    "fmd_matris_line_envelope": [_P, _I64, _P, _I64, _I64, _I32, _P, _I64, _P, _P],
    "fmd_matris_line_envelope_bwd": [_P, _I64, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _P, _I64, _P],
    "fmd_matris_forces": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, c_double, _P, _P, _P,
                          _P, _P],
    "fmd_mace_edge_geometry": [_P, _P, _P, _P, _I64, c_float, _I32, _I32, _P, _P, _P],
    "fmd_mace_edge_geometry_bwd": [_P, _P, _P, c_float, _I32, _I32, _P, _P, _P, _P, _I64, _P, c_float, _I32, _P],
    "fmd_mace_edge_virial": [_P, _P, _P, c_float, _I32, _I32, _P, _I64, _P, _P, c_float, _P, _P, _I32, _P],
    "fmd_mace_message": [_P, _I32, _P, _P, _P, _P, _P, _I64, _I32, c_float, _P, _P, _P],
    "fmd_mace_message_bwd": [_P, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, c_float, _P, _P, _I32, _P, _P,
                             _P],
    "fmd_mace_product": [_P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P],
    "fmd_mace_product_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P],
    "fmd_element_linear": [_P, _I64, _I32, _P, _P, _I32, _I32, _I32, _P, _I32, _P],
    "fmd_mace_node_energy": [_P, _I32, _I64, _P, _P, c_double, c_double, _I64, _I32, _P, _P, _P],
    "fmd_mace_node_energy_bwd": [_P, c_double, _I64, _I32, _P, _P],
    "fmd_nequip_edge_basis": [_P, _P, _P, _P, _P, _P, _I64, c_float, _I32, _I32, _P, _P, _P, _P],
    "fmd_nequip_edge_basis_bwd": [_P, _P, _P, _P, _P, _I64, c_float, _I32, _I32, _P, _P],
    "fmd_nequip_conv": [_P, _P, _P, _P, _P, _P, _I64, c_float, _P, _P],
    "fmd_nequip_conv_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, c_float, _P, _P, _P, _P, _I32, _P],
    "fmd_edge_forces": [_P, _P, _P, _P, _P, _I64, _P, _P],
    "fmd_zero": [_P, _I64, _P],
    "fmd_nequip_self_connection": [_P, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P],
    "fmd_nequip_gate": [_P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P],
    "fmd_nequip_gate_bwd": [_P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P],
    "fmd_nhc_pre_force": [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P],
    "fmd_nhc_post_pre_force": [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P],
    "fmd_nhc_post_force": [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _P],
}
_RESTYPES = {"fmd_status_string": ctypes.c_char_p, "fmd_last_error": ctypes.c_char_p}

_lib = None


def declare(name: str, argtypes: list, restype=c_int32) -> None:
    """Register the signature of an entry point (used by modules that add kernels)."""
    _SIGNATURES[name] = argtypes
    if restype is not c_int32:
        _RESTYPES[name] = restype
    if _lib is not None:
        _bind(_lib, name)


def _bind(lib, name: str) -> None:
    fn = getattr(lib, name)
    fn.argtypes = _SIGNATURES[name]
    fn.restype = _RESTYPES.get(name, c_int32)


def lib():
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise FastMDLibraryError(
                f"{LIBRARY} is not built: run `python -m fastmd_b200.build` (nvcc, sm_100a)")
        try:
            handle = ctypes.CDLL(str(LIBRARY))
        except OSError as error:
            raise FastMDLibraryError(f"cannot load {LIBRARY}: {error}") from error
        for name in _SIGNATURES:
            _bind(handle, name)
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        text = lib().fmd_status_string(status).decode()
        detail = lib().fmd_last_error().decode() if status == 2 else ""
        raise FastMDLibraryError(f"{what}: {text}" + (f" ({detail})" if detail else ""))


# kernels each entry point launches (for the launch count of a step); the default is one
KERNELS_PER_CALL = {"fmd_refilter_edges": 2, "fmd_refilter_edges_noalloc": 2, "fmd_mace_message_bwd": 2,
                    "fmd_mace_edge_virial": 2, "fmd_reverse_pairs": 5, "fmd_line_graph": 6, "fmd_column_sum": 2}


def fused_step_kernels(n_layers: int) -> int:
    """Launches of one fmd_mace_fused_step: edge_fwd, L messages, L-1 node_fwd, node_last,
    L-1 (msg_bwd_edge + sender_node), msg_bwd_edge(0), edge_bwd, forces."""
    return 1 + n_layers + (n_layers - 1) + 1 + 2 * (n_layers - 1) + 1 + 1 + 1
_counting: dict | None = None


def count_launches(enabled: bool = True) -> dict | None:
    """Start (or stop and return) counting entry-point calls made through ``call``."""
    global _counting
    if enabled:
        _counting = {}
        return None
    counted, _counting = _counting, None
    return counted


def call(name: str, *args) -> None:
    if _counting is not None:
        _counting[name] = _counting.get(name, 0) + 1
    check(getattr(lib(), name)(*args), name)


def ptr(tensor) -> int | None:
    """The device address of ``tensor`` (None for None)."""
    if tensor is None:
        return None
    return tensor.data_ptr()


def stream(device=None) -> int:
    """The handle of torch's current CUDA stream (kernels are launched on it)."""
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise FastMDLibraryError("fastmd_b200 kernels run on CUDA tensors only (no CPU fallback)")


_flags: dict[int, torch.Tensor] = {}


def flags_word(device) -> torch.Tensor:
    """The per-device int32 flags word the op kernels raise FMD_FLAG_* bits in."""
    index = torch.device(device).index
    index = torch.cuda.current_device() if index is None else index
    word = _flags.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=f"cuda:{index}")
        _flags[index] = word
    return word


c_int32_t, c_int64_t = c_int32, c_int64
c_void_p_t = c_void_p

__all__ = ["FastMDLibraryError", "FmdCatPart", "call", "check", "declare", "flags_word", "lib", "ptr",
           "require_cuda", "stream", "c_double", "c_float", "c_int32", "c_int64", "c_void_p", "ctypes"]
