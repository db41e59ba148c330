"""The C-ABI library loads, exports every declared entry point, and its host-only
functions (status mapping, defaults, lr schedule) agree with the oracle.
No kernel is launched here; these run without a GPU."""
from __future__ import annotations

import ctypes
import re
import struct
from pathlib import Path

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "slmopt.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(slm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(names) <= bound | {"slm_opt_handle"}, set(names) - bound


def test_status_codes_and_categories():
    lib = _lib.load()
    expect = {
        0: ("OK", 0),
        10: ("MODEL_GRADIENT_NONFINITE", 5),
        11: ("MODEL_GRADIENT_NORM_NONFINITE", 5),
        12: ("MODEL_OPTIMIZER_INPUT_INVALID", 5),
        13: ("MODEL_OPTIMIZER_RESULT_NONFINITE", 5),
        20: ("P12_OPTIMIZER_GRADIENT_INVALID", 3),
        21: ("P12_SCHEDULER_STATE_MISMATCH", 3),
        22: ("P12_OPTIMIZER_STATE_INVALID", 3),
        23: ("P12_UPDATE_INDEX_INVALID", 3),
        24: ("P12_SCHEDULE_INDEX_INVALID", 3),
        26: ("E1_STATE_ARTIFACT_INVALID", 3),
        30: ("SLM_INVALID_ARGUMENT", 2),
        40: ("SLM_CUDA_ERROR", 4),
        43: ("SLM_TIMEOUT", 4),
        50: ("SLM_INTERNAL_ERROR", 1),
    }
    for status, (code, cat) in expect.items():
        assert lib.slm_status_code_string(status).decode() == code
        assert lib.slm_status_category(status) == cat
    # oracle and product share the numbering
    assert oracle.MODEL_GRADIENT_NONFINITE == _lib.SLM_ERR_MODEL_GRADIENT_NONFINITE
    assert oracle.P12_SCHEDULER_STATE_MISMATCH == _lib.SLM_ERR_P12_SCHEDULER_STATE_MISMATCH


def test_struct_layouts_match_oracle():
    assert ctypes.sizeof(_lib.StepConfig) == ctypes.sizeof(oracle.StepConfig) == 56
    assert ctypes.sizeof(_lib.StepResult) == ctypes.sizeof(oracle.StepResult)
    assert [f for f, _ in _lib.StepResult._fields_] == [f for f, _ in oracle.StepResult._fields_]


def test_learning_rate_schedules_bit_equal_to_oracle():
    lib = _lib.load()
    out = ctypes.c_float()
    for t in list(range(1, 2001)) + list(range(2001, 30519, 97)) + [30518]:
        st = lib.slm_canonical_learning_rate(t, ctypes.byref(out))
        ost, olr = oracle.canonical_learning_rate(t)
        assert st == ost == 0
        assert struct.pack("<f", out.value) == struct.pack("<f", olr), t
    assert lib.slm_canonical_learning_rate(0, ctypes.byref(out)) == \
        _lib.SLM_ERR_P12_SCHEDULE_INDEX_INVALID
    assert lib.slm_canonical_learning_rate(30519, ctypes.byref(out)) == \
        _lib.SLM_ERR_P12_SCHEDULE_INDEX_INVALID
    for t in range(1, 101):
        st = lib.slm_schedule_learning_rate(t, 3e-4, 3e-5, 20, 100, ctypes.byref(out))
        assert st == 0
        assert np.float32(out.value) == np.float32(oracle.schedule_learning_rate(
            t, 3e-4, 3e-5, 20, 100)[1])


def test_create_without_device_fails_cleanly():
    from conftest import have_gpu

    if have_gpu():
        pytest.skip("a GPU is visible")
    from slmopt import B200Adamw, SlmError, TensorTable

    with pytest.raises(SlmError) as e:
        B200Adamw(TensorTable.from_sizes([8]))
    assert e.value.code == "SLM_NO_DEVICE" and e.value.category == 4


def test_create_rejects_bad_tables_before_touching_a_device():
    lib = _lib.load()
    h = ctypes.c_void_p()
    assert lib.slm_opt_create(None, 0, 0, ctypes.byref(h)) == _lib.SLM_ERR_P12_OPTIMIZER_STATE_INVALID


def test_every_handle_entry_point_rejects_null_arguments():
    # argument checks come before any device work, so these run without a GPU
    lib = _lib.load()
    cfg = _lib.StepConfig()
    lib.slm_step_config_default(ctypes.byref(cfg))
    res = _lib.StepResult()
    i, u32, u64 = ctypes.c_int(), ctypes.c_uint32(), ctypes.c_uint64()
    f, p, d = ctypes.c_float(), ctypes.c_void_p(), (ctypes.c_double * 8)()
    buf = ctypes.create_string_buffer(128)
    one = ctypes.c_float(1.0)
    calls = {
        "slm_opt_init_master": (None, None, None),
        "slm_opt_snapshot": (None, 0, None, 0),
        "slm_opt_restore": (None, 0, None, 0),
        "slm_opt_validate_state": (None,),
        "slm_opt_device_buffer": (None, 0, ctypes.byref(p)),
        "slm_opt_state_sha256": (None, buf),
        "slm_opt_step": (None, None, 1, 0, ctypes.byref(cfg), ctypes.byref(res), None),
        "slm_opt_read_result": (None, ctypes.byref(res)),
        "slm_opt_upload_gradients": (None, None, 1, ctypes.byref(i)),
        "slm_opt_step_uploaded": (None, 0, ctypes.byref(cfg), None, None),
        "slm_opt_norm_pass": (None, None, 1, 0, ctypes.byref(cfg), None),
        "slm_opt_update_pass": (None, ctypes.byref(cfg), None),
        "slm_opt_norm_pass_accumulate": (None, None, None, 1, 0, 0, ctypes.byref(cfg), None),
        "slm_opt_apply_update": (None, None, 0, ctypes.c_float(3e-4), 1, 0, None),
        "slm_opt_shard_range": (None, ctypes.byref(u64), ctypes.byref(u64)),
        "slm_opt_zero1_set_exchange": (None, 0),
        "slm_opt_gradient_buffer": (None, ctypes.byref(p), ctypes.byref(u64)),
        "slm_opt_set_loss_scale": (None, one, 0),
        "slm_opt_get_loss_scale": (None, ctypes.byref(f), ctypes.byref(u32)),
        "slm_opt_export_weights_f32": (None, None, 0, None),
        "slm_opt_phase_timing": (None, 1),
        "slm_opt_phase_times": (None, d, 8, ctypes.byref(u32), ctypes.byref(u64)),
        "slm_grad_accumulate": (None, None, 1, 0, 0, None),
        "slm_grad_norm_noalloc": (None, 1, 10, one, one, None, None),
        "slm_gradient_clip_scale": (None, 10, None, None),
        "slm_gradient_clip_scale_ws": (None, 10, None, 0, None, None),
    }
    for name, args in calls.items():
        assert getattr(lib, name)(*args) == _lib.SLM_ERR_INVALID_ARGUMENT, name
        assert lib.slm_last_error_message().decode() != "no error", name
    assert lib.slm_opt_destroy(None) == _lib.SLM_OK  # like free(NULL)
    assert lib.slm_opt_phase_name(None, 0) is None


def test_noalloc_norm_rejects_misaligned_pointers_before_touching_a_device():
    # A misaligned gradient or result pointer would fault the caller's context
    # inside the kernel; the entry point refuses it first (no GPU needed).
    lib = _lib.load()
    one = ctypes.c_float(1.0)
    aligned = 0x10000
    cases = [
        (aligned + 2, _lib.DTYPE_F32, aligned),   # f32 gradients 2 bytes off
        (aligned + 1, _lib.DTYPE_BF16, aligned),  # bf16 gradients 1 byte off
        (aligned, _lib.DTYPE_F32, aligned + 4),   # result not 8-byte aligned
    ]
    for grads, dtype, out in cases:
        st = lib.slm_grad_norm_noalloc(grads, dtype, 16, one, one, out, None)
        assert st == _lib.SLM_ERR_INVALID_ARGUMENT, (grads, dtype, out)
        assert "align" in lib.slm_last_error_message().decode()


def test_clip_workspace_size_and_validation_without_a_device():
    # 29 bytes per 8,192-gradient window (f64 sum, i32 base binade, four u32
    # totals, one flag byte), rounded up to 16; a workspace that is smaller or
    # misaligned is refused before any launch.
    lib = _lib.load()
    assert lib.slm_gradient_clip_workspace_bytes(0) == 0
    assert lib.slm_gradient_clip_workspace_bytes(1) == 32
    assert lib.slm_gradient_clip_workspace_bytes(8192) == 32
    assert lib.slm_gradient_clip_workspace_bytes(8193) == 64
    assert lib.slm_gradient_clip_workspace_bytes(135_285_504) == 478_944  # 16,515 windows
    need = lib.slm_gradient_clip_workspace_bytes(10 * 8192)
    grads, ws, out = 0x10000, 0x20000, 0x30000
    st = lib.slm_gradient_clip_scale_ws(grads, 10 * 8192, ws, need - 16, out, None)
    assert st == _lib.SLM_ERR_INVALID_ARGUMENT
    assert "workspace" in lib.slm_last_error_message().decode()
    st = lib.slm_gradient_clip_scale_ws(grads, 10 * 8192, ws + 8, need, out, None)
    assert st == _lib.SLM_ERR_INVALID_ARGUMENT
    assert "align" in lib.slm_last_error_message().decode()


def test_staging_copy_is_exact_at_every_alignment_and_size():
    # The host copy that fills the pinned staging ring (non-temporal stores for
    # large copies where the CPU has AVX2) must move every byte, whatever the
    # alignment of either side and whatever the tail.
    import numpy as np

    lib = _lib.load()
    fn = getattr(lib, "_ZN6slmopt11stream_copyEPvPKvm")
    fn.restype = None
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    rng = np.random.default_rng(4)
    src = rng.integers(0, 256, (1 << 20) + 300, dtype=np.uint8)
    for n in (0, 1, 31, 4096, (1 << 16) - 1, 1 << 16, (1 << 16) + 77, (1 << 20) + 129):
        for so, do in ((0, 0), (1, 0), (0, 7), (13, 29), (32, 5)):
            dst = np.zeros(n + 64, np.uint8)
            fn(dst.ctypes.data + do, src.ctypes.data + so, n)
            assert np.array_equal(dst[do:do + n], src[so:so + n]), (n, so, do)
            assert not dst[:do].any() and not dst[do + n:].any(), (n, so, do)


def test_c_caller_compiles_against_the_header_and_links(tmp_path):
    # The header is the binding's source of truth for Go / Rust / Java: it
    # must compile as strict C11, and a C program must link and call the
    # library (entry points that need no GPU).
    import shutil
    import subprocess

    from slmopt import build

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lib = _lib.library_path()
    exe = tmp_path / "abi_caller"
    src = Path(__file__).with_name("abi_caller.c")
    cmd = [gcc, "-std=c11", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(build.INCLUDE),
           str(src), "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
