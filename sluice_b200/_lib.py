"""ctypes binding of the C ABI (``include/sluice_b200.h``).

The library ``libsluice_sm100.so`` is built in-tree by
``python -m sluice_b200.csrc.build``. There is no fallback: every op in this
package raises if the library is missing or a call fails.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsluice_sm100.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "sluice_b200.h")

SL_OK = 0
SL_ERR_OVERFLOW = 1
SL_ERR_INVALID = 2
SL_ERR_CUDA = 3
SL_ERR_UNSUPPORTED = 4
SL_ERR_TIMEOUT = 5
SL_ERR_NO_SCRATCH = 6

SEG_FREE, SEG_PROBATION, SEG_PROTECTED, SEG_PINNED = 0, 1, 2, 3
PLAN_FAST_HIT = 1
PLAN_LFU = 2
# parts of a phased fused-experts call (include/sluice_b200.h SL_PHASE_*)
PHASE_GROUP, PHASE_RESIDENT_GEMMS, PHASE_STREAMED_GEMMS, PHASE_COMBINE = 2, 3, 4, 5

# state header words / counters (include/sluice_b200.h)
HDR = dict(num_slots=0, global_n=1, local_n=2, protected_cap=3, flags=4,
           map_is_standing=5, free_top=6, protected_count=7, clock=8, status=9,
           fill_count=10, last_misses=11, lfu_steps=12, prefetch_fills=13)
CNT = dict(gaps=0, fast_hits=1, misses=2, hits=3, overflows=4, fills=5, scan_steps=6,
           scan_hits=7, scan_misses=8, waves=9, prefetches=10)
STATE_NFIELDS = 12
NUM_COUNTERS = 16

# wave plan header words (sl_plan_waves)
WAVE_HDR = dict(num_waves=0, status=1, max_waves=2, global_n=3, num_slots=4, leftover=5,
                rotation=6)
WAVE_NFIELDS = 5

_c = ctypes
_vp, _i, _sz, _f = _c.c_void_p, _c.c_int, _c.c_size_t, _c.c_float

WEIGHTS_BF16, WEIGHTS_FP8_BLOCK128 = 0, 1


class ExpertWeights(ctypes.Structure):
    """``sl_expert_weights`` (include/sluice_b200.h)."""

    _fields_ = [("w13", _vp), ("w2", _vp), ("w13_scale", _vp), ("w2_scale", _vp),
                ("num_slots", _i), ("shared_w13", _vp), ("shared_w2", _vp),
                ("shared_w13_scale", _vp), ("shared_w2_scale", _vp), ("n_shared", _i),
                ("dtype", _i)]


_SIGNATURES = {
    "sl_status_string": (_c.c_char_p, [_i]),
    "sl_version": (_i, []),
    "sl_device_sm_count": (_i, []),
    "sl_route": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp,
                      _vp, _vp, _vp]),
    "sl_gate": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "sl_select_experts": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp,
                               _vp]),
    "sl_slot_state_bytes": (_sz, [_i, _i, _i]),
    "sl_slot_state_offsets": (_i, [_i, _i, _i, _vp]),
    "sl_slot_state_init": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i,
                                _vp]),
    "sl_plan_slots": (_i, [_vp, _vp, _i, _vp, _vp]),
    "sl_prefetch_slots": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "sl_stream_experts": (_i, [_vp, _i, _vp, _vp, _vp, _i, _vp]),
    "sl_stream_experts_strided": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "sl_wave_plan_bytes": (_sz, [_i, _i, _i]),
    "sl_wave_plan_offsets": (_i, [_i, _i, _i, _vp]),
    "sl_wave_plan_init": (_i, [_vp, _i, _i, _i, _vp]),
    "sl_plan_waves": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp, _vp]),
    "sl_stream_wave": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "sl_host_alloc_mapped": (_i, [_sz, _c.POINTER(_vp)]),
    "sl_host_free": (_i, [_vp]),
    "sl_fused_experts_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "sl_fused_experts": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i, _vp,
                              _i, _vp, _vp, _i, _f, _vp, _vp, _sz, _vp]),
    "sl_fused_experts_phase": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i, _vp,
                                    _i, _vp, _vp, _i, _f, _vp, _i, _vp, _vp, _sz, _vp]),
    "sl_fused_experts_partial": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i,
                                      _vp, _i, _vp, _vp, _i, _i, _i, _f, _vp, _vp, _sz,
                                      _vp]),
    "sl_fused_experts_ex": (_i, [_vp, _i, _i, _i, _c.POINTER(ExpertWeights), _vp, _vp, _i,
                                 _vp, _i, _f, _i, _i, _vp, _i, _i, _vp, _vp, _sz, _vp]),
    "sl_ep_dispatch_recv_bytes": (_sz, [_i, _i, _i, _i]),
    "sl_ep_combine_recv_bytes": (_sz, [_i, _i, _i]),
    "sl_ep_dispatch": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                            _vp, _vp, _vp, _vp]),
    "sl_ep_combine": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                           _vp, _vp]),
    "sl_fused_experts_noalloc": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i,
                                      _vp, _i, _vp, _vp, _i, _f, _vp, _vp, _vp]),
    "sl_add_rmsnorm": (_i, [_vp, _vp, _vp, _f, _vp, _i, _i, _vp]),
    "sl_linear_small": (_i, [_vp, _i, _i, _vp, _i, _vp, _vp]),
    "sl_mla_decode": (_i, [_vp, _i, _vp, _f, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                           _i, _i, _f, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


class SluiceError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int):
        self.status = status
        super().__init__(f"{what}: {status_text(status)} (status {status})")


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sl_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load the library once; raise loudly if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m sluice_b200.csrc.build` (nvcc, sm_100a). "
                    "sluice_b200 has no CPU fallback.")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def status_text(status: int) -> str:
    try:
        return lib().sl_status_string(int(status)).decode()
    except Exception:  # library not loadable: plain text
        return {0: "ok", 1: "overflow", 2: "invalid argument", 3: "CUDA error",
                4: "unsupported", 5: "timeout",
                6: "problem too large for the no-alloc scratch"}.get(int(status), "unknown")


def check(rc: int, what: str) -> None:
    if rc != SL_OK:
        raise SluiceError(what, rc)


def ptr(t) -> int | None:
    """Raw data pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
