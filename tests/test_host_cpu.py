"""CPU tier: the C-ABI library loads and exports its header, and the host-side
logic (initial slot residency, state layout) matches the oracle."""

import ctypes
import json
import os

import pytest

from oracle.slot_policy import PINNED, SlotPolicyModel
from sluice_b200 import _lib
from sluice_b200.offloader import initial_slot_state, protected_cap_for

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = _lib.header_symbols()
    assert len(syms) >= 12
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(_lib._SIGNATURES) == set(syms)


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.sl_version() >= 100
    assert b"raise SLUICE_SLOTS" in L.sl_status_string(_lib.SL_ERR_OVERFLOW)
    assert L.sl_status_string(_lib.SL_OK) == b"ok"


def test_state_layout_is_aligned_and_sized():
    L = _lib.lib()
    for S, G, Lc in [(48, 64, 64), (96, 128, 128), (24, 64, 32), (1, 1, 1), (1024, 4096, 256)]:
        offs = (ctypes.c_size_t * (_lib.STATE_NFIELDS + 1))()
        assert L.sl_slot_state_offsets(S, G, Lc, offs) == 0
        o = list(offs)
        assert all(v % 16 == 0 for v in o)
        assert o == sorted(o)
        assert o[-1] == L.sl_slot_state_bytes(S, G, Lc)
        assert o[3] - o[2] >= 4 * G and o[6] - o[5] >= 4 * S and o[7] - o[6] >= S


def test_host_calls_reject_bad_arguments_without_a_gpu():
    L = _lib.lib()
    assert L.sl_slot_state_bytes(0, 4, 4) == 0
    assert L.sl_fused_experts_workspace_bytes(8, 6, 2048, 1408, 48, 2) > 0
    # argument checks run before any CUDA call
    assert L.sl_route(None, None, None, 1, 100, 64, 6, 0, 1, 1, 0, 1.0, None, None, None,
                      None, None) == _lib.SL_ERR_UNSUPPORTED
    assert L.sl_select_experts(None, 4, 48, 6, 0, 1, 1, 0, 1.0, None, None, None,
                               None) == _lib.SL_ERR_UNSUPPORTED  # E % 32
    assert L.sl_fused_experts(None, 4, 2048, 1400, None, None, 8, 0, None, None, 2, None,
                              0, None, None, 0, 1.0, None, None, 0, None) == _lib.SL_ERR_UNSUPPORTED
    assert L.sl_fused_experts(None, 4, 2048, 1408, None, None, 8, 1, None, None, 2, None,
                              0, None, None, 0, 1.0, None, None, 0, None) == _lib.SL_ERR_UNSUPPORTED
    assert L.sl_plan_slots(None, None, 0, None, None) == _lib.SL_ERR_INVALID
    assert L.sl_stream_experts(None, 0, None, None, None, 0, None) == _lib.SL_ERR_INVALID
    assert L.sl_stream_experts_strided(None, 0, None, None, None, None, 0,
                                       None) == _lib.SL_ERR_INVALID
    # expert-parallel exchange: sizes, and world / rank / shape checks
    # routed rows: hidden | weights | ids | token index, padded to 16 bytes,
    # after a 128-byte header (the row counts) per half
    row = (2 * 2048 + 8 * 6 + 4 + 15) // 16 * 16
    assert L.sl_ep_dispatch_recv_bytes(2, 8, 2048, 6) == 2 * (128 + 2 * 8 * row)
    assert L.sl_ep_combine_recv_bytes(2, 8, 2048) == 2 * 2 * 8 * 2048 * 4
    assert L.sl_ep_dispatch_recv_bytes(0, 8, 2048, 6) == 0
    assert L.sl_ep_dispatch(None, None, None, 8, 2048, 6, 64, 0, 9, None, None, None, None,
                            None, None, None, None, None) == _lib.SL_ERR_INVALID
    assert L.sl_ep_combine(None, None, None, 8, 2048, 6, 64, 0, 0, None, None, None, None,
                           None, None, None) == _lib.SL_ERR_INVALID
    # expert waves: layout and argument checks
    offs = (ctypes.c_size_t * (_lib.WAVE_NFIELDS + 1))()
    assert L.sl_wave_plan_offsets(48, 64, 7, offs) == 0
    assert list(offs) == [0, 64, 96, 96 + 7 * 48 * 4, 96 + 2 * 7 * 48 * 4,
                          96 + 2 * 7 * 48 * 4 + 7 * 64 * 4]
    assert L.sl_wave_plan_bytes(48, 64, 7) == offs[_lib.WAVE_NFIELDS]
    assert all(v % 16 == 0 for v in offs)
    assert L.sl_wave_plan_bytes(0, 64, 7) == 0 and L.sl_wave_plan_bytes(48, 64, 0) == 0
    assert L.sl_wave_plan_offsets(48, 64, 0, offs) == _lib.SL_ERR_INVALID
    assert L.sl_wave_plan_init(None, 48, 64, 7, None) == _lib.SL_ERR_INVALID
    assert L.sl_plan_waves(None, None, 8, 6, 0, None, None, None) == _lib.SL_ERR_INVALID
    assert L.sl_stream_wave(None, 0, 2, None, None, None, None, 0, None) == _lib.SL_ERR_INVALID
    # fp8 through the general entry without weights or block scales: refused
    # before anything is dereferenced
    w = _lib.ExpertWeights()
    w.num_slots, w.dtype = 8, 1  # SL_WEIGHTS_FP8_BLOCK128
    assert L.sl_fused_experts_ex(None, 4, 2048, 1408, ctypes.byref(w), None, None, 2, None, 0,
                                 1.0, 0, -1, None, -1, 0, None, None, 0, None) \
        == _lib.SL_ERR_INVALID
    # phased calls: phases 0..5 only (-1, the whole call, is sl_fused_experts)
    for bad in (-1, 6):
        assert L.sl_fused_experts_phase(None, 4, 2048, 1408, None, None, 8, 0, None, None, 2,
                                        None, 0, None, None, 0, 1.0, None, bad, None, None, 0,
                                        None) == _lib.SL_ERR_INVALID
    w.dtype = 0
    assert L.sl_fused_experts_ex(None, 4, 2048, 1408, ctypes.byref(w), None, None, 2, None, 0,
                                 1.0, 0, -1, None, _lib.PHASE_COMBINE + 1, 0, None, None, 0,
                                 None) == _lib.SL_ERR_INVALID
    # the decoder harness's kernels: shapes outside their lane layouts and
    # missing buffers are refused before any CUDA call
    mla = lambda rank, rope: L.sl_mla_decode(None, 16 * 192 + rank + rope, None, 1e-6, None,
                                             None, None, None, None, 8, 16, 128, rope, rank,
                                             128, 384, 0.07, None, None)
    assert mla(256, 64) == _lib.SL_ERR_UNSUPPORTED     # the latent width is fixed at 512
    assert mla(512, 48) == _lib.SL_ERR_UNSUPPORTED     # rope a multiple of 32, at most 64
    assert mla(512, 64) == _lib.SL_ERR_INVALID         # null buffers
    assert L.sl_add_rmsnorm(None, None, None, 1e-6, None, 8, 2044, None) == _lib.SL_ERR_INVALID
    assert L.sl_add_rmsnorm(None, None, None, 1e-6, None, 8, 16384, None) == _lib.SL_ERR_INVALID
    assert L.sl_add_rmsnorm(None, None, None, 1e-6, None, 0, 2048, None) == _lib.SL_OK
    assert L.sl_linear_small(None, 5, 2048, None, 64, None, None) == _lib.SL_ERR_INVALID
    assert L.sl_linear_small(None, 1, 2044, None, 64, None, None) == _lib.SL_ERR_INVALID
    assert L.sl_linear_small(None, 0, 2048, None, 64, None, None) == _lib.SL_OK


@pytest.mark.parametrize("S,frac", [(48, 0.5), (48, 0.0), (48, 0.95), (1, 0.5), (96, 0.9)])
def test_protected_cap_matches_oracle(S, frac):
    m = SlotPolicyModel(S, list(range(S + 4)), S + 4, protect_frac=frac)
    assert protected_cap_for(S, frac) == m.protected_cap


def _scenarios():
    with open(os.path.join(GOLDEN, "slot_traces.json")) as f:
        return json.load(f)["scenarios"]


@pytest.mark.parametrize("sc", _scenarios(), ids=lambda s: s["name"])
def test_initial_state_matches_oracle(sc):
    init = initial_slot_state(sc["num_slots"], sc["local_of"], sc["local_n"],
                              sc["protect_frac"], sc["pins"], sc["prefill_resident"])
    m = SlotPolicyModel(sc["num_slots"], sc["local_of"], sc["local_n"],
                        protect_frac=sc["protect_frac"],
                        prefill_resident=sc["prefill_resident"])
    if sc["pins"]:
        m.apply_pins(sc["pins"])
    assert init.protected_cap == m.protected_cap == sc["protected_cap"]
    assert init.expert_in_slot == m.expert_in_slot
    assert init.free_stack == m.free_stack
    assert [s for s in range(m.num_slots) if init.seg[s] == PINNED] == \
        [s for s in range(m.num_slots) if m.seg[s] == PINNED]
    if sc["pins"]:
        assert sorted(s for _, s in init.fills) == sc["pinned_slots"]


def test_pin_file_formats(tmp_path):
    """SLUICE_PIN_FILE: {"layers": {ordinal: ids}} or the bare mapping;
    malformed files fail loudly (the reference refuses a silent empty pin)."""
    import json

    import pytest as _pytest

    from sluice_b200.offloader import load_pin_file

    a = tmp_path / "a.json"
    a.write_text(json.dumps({"layers": {"0": [3, 5], "2": ["7"]}}))
    assert load_pin_file(str(a)) == {0: [3, 5], 2: [7]}
    b = tmp_path / "b.json"
    b.write_text(json.dumps({"1": [9]}))
    assert load_pin_file(str(b)) == {1: [9]}
    c = tmp_path / "c.json"
    c.write_text("{not json")
    with _pytest.raises(ValueError):
        load_pin_file(str(c))
    with _pytest.raises(OSError):
        load_pin_file(str(tmp_path / "missing.json"))


def test_lfu_changes_victims_only_when_counts_differ():
    """Oracle: with every count equal the LFU order is the LRU order, so an
    LFU cache fed one expert per step behaves exactly like the plain SLRU."""
    from oracle.slot_policy import SlotPolicyModel

    lru = SlotPolicyModel(4, list(range(16)), 16)
    lfu = SlotPolicyModel(4, list(range(16)), 16, lfu=True)
    for g in [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]:
        assert lru.gap([g]) == lfu.gap([g])
        assert lru.snapshot()["expert_in_slot"] == lfu.snapshot()["expert_in_slot"]


def test_reference_arm_runs_the_global_batch(monkeypatch, capsys):
    """`bench.py --impl reference` under torchrun at N=2: rank 0 times the CPU
    port on the GPU arm's global batch (c x N tokens, beyond the slot
    envelope, so in envelope-sized chunks) and prints one JSON line."""
    import json
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench

    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "2")
    argv = ["--impl", "reference", "--steps", "1", "--warmup", "1", "--layers", "2"]
    bench.main(argv)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["config"]["global_batch"] == 16 and line["value"] > 0
    assert "c=16" in line["cpu_baseline"]["sample"]
    # the same config dict the GPU arm prints for these arguments at N=2
    # (24 of 32 local experts in slots per rank)
    from sluice_b200 import configs
    a = bench._args(argv[2:])
    cfg = configs.CONFIGS[a.config]
    assert line["config"] == bench._config(a, cfg, bench._slots_for(a, cfg, 2), 8, 2, 2)
    assert line["config"]["slots"] == 24 and line["config"]["slots_frac"] == 0.75


def test_cpu_port_plans_steps_beyond_the_envelope_in_waves():
    """The CPU port (the reference arm and the CPU baselines) runs a step of
    more than slots // topk tokens as the reference's classic hook does:
    one wave plan over the whole step, no chunking."""
    import os
    import sys

    import torch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    from sluice_b200 import configs

    cfg = configs.V2_LITE
    run = bench.cpu_layer_runner(cfg, seed=0, n_weight_sets=1)
    x = torch.randn(24, cfg.hidden, generator=torch.Generator().manual_seed(1))
    out = run(0, x.to(torch.bfloat16), 48, False)
    pol = run.policies[0]
    assert out.shape == (24, cfg.hidden) and torch.isfinite(out.float()).all()
    assert pol.scan_steps == 1 and pol.gaps == 0 and pol.scan_waves >= 1
    run(0, x[:8].to(torch.bfloat16), 48)          # within the envelope: the gap
    assert pol.gaps == 1 and pol.scan_steps == 1


def test_bench_launch_count_rule():
    """gpu_launches per layer: resident 6 (gate, select, grouping, 2 GEMMs,
    combine), offloaded 10 (+ plan, stream, both GEMMs again), serial gap 8,
    +1 quantising gather for fp8, +2 exchange kernels; a step beyond the
    envelope: plan + one stream per wave + wave 0 in two phases + later
    waves as whole calls."""
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    from sluice_b200 import configs
    from sluice_b200.offloader import max_waves_for

    V2, V3 = configs.V2_LITE, configs.DEEPSEEK_V3
    assert bench.layer_launches(V2, 8, 1, 64) == 6
    assert bench.layer_launches(V2, 8, 1, 48) == 10
    assert bench.layer_launches(V2, 8, 1, 48, no_overlap=True) == 8
    assert bench.layer_launches(V2, 8, 2, 48) == 8
    assert bench.layer_launches(V2, 8, 2, 48, exchange="nccl") == 6
    # the decoder harness's own kernels: first RMSNorm, per layer MLA + two
    # add + RMSNorm, plus the two projections for one or two rows
    assert bench.harness_launches(27, 8) == 1 + 27 * 3
    assert bench.harness_launches(27, 1) == 1 + 27 * 5
    assert bench.layer_launches(V3, 8, 8, 128) == 9
    mw = max_waves_for(48, 64, 24, 0)
    assert bench.layer_launches(V2, 512, 1, 48, decode=False) == 2 + 1 + mw + 7 + \
        (mw - 1) * 5 == 35
    # decode steps beyond the envelope: every expert decode-class, fewer waves
    mwd = max_waves_for(96, 128, 48, 0, all_decode=True)
    assert mwd == 3 < max_waves_for(96, 128, 48, 0) == 5
    assert bench.layer_launches(V3, 8, 2, 96) == 2 + 1 + mwd + 7 + (mwd - 1) * 5 + 2


def test_decode_rows_from_query_start_loc_matches_the_reference():
    """The host helper that turns a non-MLA backend's attention metadata into
    decode rows, against the reference's own ``_non_mla_decode_rows`` on the
    same metadata (tests/golden/nonmla_rows.json)."""
    import torch

    from sluice_b200.layer import decode_rows_from_query_start_loc

    with open(os.path.join(GOLDEN, "nonmla_rows.json")) as f:
        cases = json.load(f)["cases"]
    assert any(c["rows"] is None for c in cases) and any(c["rows"] == [] for c in cases)
    for c in cases:
        got = decode_rows_from_query_start_loc(torch.tensor(c["query_start_loc"]),
                                               c["num_tokens"], c["max_query_len"],
                                               c["num_actual_tokens"])
        assert (None if got is None else got.tolist()) == c["rows"], c


def test_plan_ids_for_orders_decode_rows_first():
    import torch

    from sluice_b200.offloader import plan_ids_for

    ids = torch.arange(12, dtype=torch.int32).view(6, 2)
    same, d = plan_ids_for(ids, 3)
    assert d == 3 and torch.equal(same, ids)
    got, d = plan_ids_for(ids, torch.tensor([4, 1, 4]))
    assert d == 2 and got[:, 0].tolist() == [2, 8, 0, 4, 6, 10]
    assert plan_ids_for(ids, [])[1] == -1             # a pure prefill: scan
    assert plan_ids_for(ids, list(range(6)))[1] == 6  # every row a decode


def _header_enum(prefix: str) -> dict:
    """Values of the header's ``prefix*`` enumerators (sequential enums with
    an explicit first value, as include/sluice_b200.h writes them)."""
    import re

    with open(_lib.HEADER_PATH) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    out = {}
    for body in re.findall(r"enum\s*\{(.*?)\}", text, flags=re.S):
        nxt = 0
        for item in [x.strip() for x in body.split(",") if x.strip()]:
            name, _, val = item.partition("=")
            name = name.strip()
            nxt = int(val.strip(), 0) if val.strip() else nxt
            if name.startswith(prefix):
                out[name[len(prefix):].lower()] = nxt
            nxt += 1
    return out


def test_binding_tables_match_the_header():
    """The ctypes binding's state-header, counter, wave-plan and status
    tables against the header's enums (a drift would misread device state)."""
    assert _header_enum("SL_HDR_") == _lib.HDR
    assert _header_enum("SL_CNT_") == _lib.CNT
    assert _header_enum("SL_WAVE_HDR_") == _lib.WAVE_HDR
    assert _header_enum("SL_STATE_NFIELDS")[""] == _lib.STATE_NFIELDS
    assert _header_enum("SL_WAVE_NFIELDS")[""] == _lib.WAVE_NFIELDS
    plan = _header_enum("SL_PLAN_")
    assert plan == {"fast_hit": _lib.PLAN_FAST_HIT, "lfu": _lib.PLAN_LFU}
    err = _header_enum("SL_ERR_")
    assert err == {"overflow": _lib.SL_ERR_OVERFLOW, "invalid": _lib.SL_ERR_INVALID,
                   "cuda": _lib.SL_ERR_CUDA, "unsupported": _lib.SL_ERR_UNSUPPORTED,
                   "timeout": _lib.SL_ERR_TIMEOUT, "no_scratch": _lib.SL_ERR_NO_SCRATCH}
    assert len(_lib.CNT) <= _lib.NUM_COUNTERS
    assert _header_enum("SL_SEG_") == {"free": _lib.SEG_FREE, "probation": _lib.SEG_PROBATION,
                                       "protected": _lib.SEG_PROTECTED,
                                       "pinned": _lib.SEG_PINNED}
    assert _header_enum("SL_WEIGHTS_") == {"bf16": _lib.WEIGHTS_BF16,
                                           "fp8_block128": _lib.WEIGHTS_FP8_BLOCK128}


def test_state_init_rejects_bad_maps_before_any_cuda_call():
    """sl_slot_state_init validates the host arrays first: two global ids
    mapped to one local expert, a local id out of range, an expert in two
    slots, or a free slot in a segment are refused (no device is touched)."""
    L = _lib.lib()
    S, G, Ln = 4, 8, 6
    arr = lambda v, t: (t * len(v))(*v)
    dummy = ctypes.create_string_buffer(L.sl_slot_state_bytes(S, G, Ln))
    ok_lof = [0, 1, 2, 3, 4, 5, -1, -1]
    eis = [-1] * S
    seg = [0] * S
    free = [3, 2, 1, 0]

    def init(lof, eis=eis, seg=seg):
        return L.sl_slot_state_init(ctypes.addressof(dummy), S, G, Ln, 1, 0,
                                    arr(lof, ctypes.c_int32), arr(eis, ctypes.c_int32),
                                    arr(seg, ctypes.c_uint8), arr(free, ctypes.c_int32),
                                    len(free), None)

    assert init([0, 1, 2, 3, 4, 0, -1, -1]) == _lib.SL_ERR_INVALID   # not injective
    assert init([0, 1, 2, 3, 4, 6, -1, -1]) == _lib.SL_ERR_INVALID   # local id >= L
    assert init(ok_lof, eis=[2, 2, -1, -1], seg=[1, 1, 0, 0]) == _lib.SL_ERR_INVALID
    assert init(ok_lof, eis=[-1, -1, -1, -1], seg=[1, 0, 0, 0]) == _lib.SL_ERR_INVALID


def test_header_compiles_as_c99_and_cxx17(tmp_path):
    """The boundary is a C ABI: a C host (cgo, a plain C loader) includes the
    header as C99, a C++ host as C++17, both warning-free."""
    import shutil
    import subprocess

    src = tmp_path / "use_header.c"
    src.write_text(f'#include "{_lib.HEADER_PATH}"\n'
                   "int main(void) { sl_expert_weights w; w.num_slots = SL_WAVE_NFIELDS;\n"
                   "  return w.num_slots + SL_CNT_WAVES + SL_ERR_NO_SCRATCH; }\n")
    for cc, args in (("gcc", ["-std=c99", "-pedantic"]), ("g++", ["-std=c++17", "-x", "c++"])):
        if shutil.which(cc) is None:
            pytest.skip(f"{cc} not available")
        r = subprocess.run([cc, *args, "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                            str(src)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_c_host_links_and_calls_the_library(tmp_path):
    """tests/c_host/abi_check.c — a C99 program linked against
    libsluice_sm100.so, as a non-Python host would be — runs the calls that
    need no GPU and exits 0."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    here = os.path.dirname(os.path.abspath(__file__))
    libdir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "abi_check"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror",
                        "-I", os.path.dirname(_lib.HEADER_PATH),
                        os.path.join(here, "c_host", "abi_check.c"), "-o", str(exe),
                        "-L", libdir, "-lsluice_sm100", f"-Wl,-rpath,{libdir}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "c host ok" in r.stdout


def test_reference_op_names_registered_with_the_reference_schema():
    """The router-split entry of the reference calls
    torch.ops.vllm.sluice_stream_gap(hs, ti, idx) (its own op, offloader.py
    2296-2331) and torch.ops.vllm.fused_experts(h, w13, w2, tw, ti,
    activation=, global_num_experts=, expert_map=) (2590-2599): both names
    resolve after register_reference_names(), with those argument names, and
    their fakes give the output's shape without running anything."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    from sluice_b200 import ops

    ops.register_reference_names()
    assert ops.register_reference_names() == []  # idempotent
    gap = torch.ops.vllm.sluice_stream_gap.default._schema
    assert [a.name for a in gap.arguments] == ["hidden_states", "topk_ids", "layer_idx"]
    assert not any(a.alias_info for a in gap.arguments)  # mutates_args=[]
    fe = torch.ops.vllm.fused_experts.default._schema
    names = [a.name for a in fe.arguments]
    assert names[:8] == ["hidden_states", "w1", "w2", "topk_weights", "topk_ids",
                         "activation", "global_num_experts", "expert_map"]
    with FakeTensorMode():
        hs = torch.empty(8, 2048, dtype=torch.bfloat16)
        ti = torch.empty(8, 6, dtype=torch.int32)
        tw = torch.empty(8, 6)
        w13 = torch.empty(48, 2816, 2048, dtype=torch.bfloat16)
        w2 = torch.empty(48, 2048, 1408, dtype=torch.bfloat16)
        emap = torch.empty(64, dtype=torch.int32)
        assert torch.ops.vllm.sluice_stream_gap(hs, ti, 0).shape == hs.shape
        out = torch.ops.vllm.fused_experts(hs, w13, w2, tw, ti, activation="silu",
                                           global_num_experts=64, expert_map=emap)
        assert out.shape == hs.shape and out.dtype == torch.bfloat16


def test_oracle_prefetch_policy():
    """The oracle's restatement of the opt-in prefetch: an empty prediction
    changes nothing; predicted residents are skipped; fills take the free
    list first, then probation slots in LRU order, never protected or pinned
    ones; at most max_fills; the standing map follows."""
    import copy

    from oracle.slot_policy import PROBATION, PROTECTED, SlotPolicyModel

    m = SlotPolicyModel(6, list(range(16)), 16, 0.5, True)
    m.gap([0, 1, 2, 3])                      # 4 slots taken, 2 free
    m.gap([0, 1])                            # 0 and 1 promoted to protected
    before = copy.deepcopy(m.__dict__)
    assert m.prefetch([], 4) == [] and m.__dict__ == before
    assert m.prefetch([0, 1, 2], 4) == []    # all resident
    fills = m.prefetch([9, 8, 7, 6, 5], 3)   # ascending: 5, 6, 7
    assert [l for l, _ in fills] == [5, 6, 7]
    assert [s for _, s in fills][:2] == [4, 5]          # the two free slots first
    prot = set(m.segment_order(PROTECTED))
    assert all(s not in prot for _, s in fills)
    assert m.segment_order(PROBATION)[-3:] == [s for _, s in fills]
    assert all(m.expert_map[g] >= 0 for g in (5, 6, 7)) and m.prefetches == 3
    # no probation slot left to take: nothing more is filled
    m2 = SlotPolicyModel(2, list(range(8)), 8, 0.5, False)   # no FAST_HIT: hits touch
    m2.gap([0, 1])
    m2.gap([0])                              # slot of 0 promoted to protected (cap 1)
    assert m2.prefetch([5, 6], 4) == [(5, m2.slot_of[5])]
    assert m2.slot_of[1] < 0 and m2.slot_of[0] >= 0
