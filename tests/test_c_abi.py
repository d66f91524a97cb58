"""The drop-in from C: the reference's own C host and header against this library.

- The reference's example host (examples/c/main.c) compiles unchanged against include/flyhigh.h and links to
  libflyhigh.so (oracle/Makefile, target _ref/c_host); without a GPU it fails cleanly through fh_last_error.
- sizeof / offsetof of every field of every struct of the reference header (FhEngineOptions, FhSessionOptions,
  FhStreamOptions, FhClassification, FhPush, FhOptions, FhPacerOptions, FhSourceFrame, FhRequest, FhTick, FhVkMemory;
  tests/c_abi/layout.c) are the same compiled against include/flyhigh.h and against the reference's
  crates/flyhigh-capi/include/flyhigh.h.
- On a GPU, the prebuilt host runs with the reference's shipped model and prints "ok": its in-between frame of an 8-px
  shift is closer to the true middle than to either source frame, with MAE < 6.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "oracle", "_ref", "c_host")
LIB = os.path.join(ROOT, "flyhigh_engine_b200", "libflyhigh.so")


def _layout(tmp_path, include_dir, tag):
    exe = str(tmp_path / f"layout_{tag}")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-I", include_dir, "-o", exe,
                    os.path.join(ROOT, "tests", "c_abi", "layout.c")], check=True)
    return subprocess.run([exe], check=True, capture_output=True, text=True).stdout


def test_option_struct_layout_matches_reference_header(tmp_path, reference_repo):
    ours = _layout(tmp_path, os.path.join(ROOT, "include"), "ours")
    ref = _layout(tmp_path, os.path.join(reference_repo, "crates", "flyhigh-capi", "include"), "ref")
    assert ours.count("\n") == 122
    assert ours == ref


def test_reference_c_host_builds_unchanged(reference_repo):
    if not os.path.exists(LIB):
        pytest.skip("libflyhigh.so is not built")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "_ref/c_host", f"REF={reference_repo}"],
                   check=True)
    assert os.path.exists(HOST)
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except ImportError:
        has_gpu = False
    if has_gpu:
        return
    # no device here: the host reports fh_engine_create's error and exits 1, without a crash
    r = subprocess.run([HOST, "models"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1, (r.returncode, r.stdout, r.stderr)
    assert r.stderr.startswith("fh_engine_create: ") and len(r.stderr.strip()) > len("fh_engine_create: ")


@pytest.mark.gpu
def test_reference_c_host_runs(reference_models):
    if not os.path.exists(HOST):
        pytest.skip("the reference's C host was not built here (oracle/Makefile _ref/c_host)")
    r = subprocess.run([HOST, reference_models], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.strip().splitlines()[-1] == "ok", r.stdout
    assert "in-between: MAE to the true middle" in r.stdout


def test_tune_table_format(tmp_path):
    """The conv autotune table's text format (csrc/tune.hpp) on the host: the reference's own round-trip case
    (crates/flyhigh-engine/tests/defaults.rs:55-63), malformed lines skipped, sorted output, this library's candidate
    bytes and the per-GPU / driver file name."""
    exe = str(tmp_path / "tune_roundtrip")
    subprocess.run(["g++", "-std=c++17", "-Wall", "-I", os.path.join(ROOT, "flyhigh_engine_b200", "csrc"), "-o", exe,
                    os.path.join(ROOT, "tests", "c_abi", "tune_roundtrip.cpp")], check=True)
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout
    assert r.stdout.count("ok ") == 11


def test_warp_calibrator_on_synthetic_play(tmp_path):
    """The camera warp's input calibration (csrc/warp_calib.hpp) on the reference's own synthetic play
    (crates/flyhigh-engine/tests/warp.rs:1-138): it finds the 45 ms lag and the gain, turns off at once for a released
    mouse and within a few frames for a menu, and the shift it applies is the gain times the counts since the input the
    frame shows."""
    exe = str(tmp_path / "warp_calib_test")
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "flyhigh_engine_b200", "csrc"), "-o",
                    exe, os.path.join(ROOT, "tests", "c_abi", "warp_calib_test.cpp")], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout
    assert r.stdout.count("\nok ") + r.stdout.startswith("ok ") == 10, r.stdout
