"""ctypes shim over libkernrelay.so with the reference's Python API.

Same functions, arguments, defaults and return convention as the reference's
python/kernrelay/libapi.py:20-132: each call returns the library's JSON result
as a dict with "_rc" added; a failing call returns {"error": ...} and a non-zero
"_rc".  KERNRELAY_LIB overrides the library path.  Buffers: 1 MiB for run
results, 4 MiB for profiles (libapi.py:60, :123).
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path

from ._lib import lib as _lib
from ._lib import lib_path  # noqa: F401  (same name as the reference module)

import ctypes


def lib():
    return _lib()


def version() -> str:
    return lib().kr_version().decode()


def _decode(buf, rc):
    try:
        payload = json.loads(buf.value.decode())
    except Exception:
        payload = {"error": buf.value.decode(errors="replace")}
    payload["_rc"] = rc
    return payload


def qwen_run(model_dir, mode="serial_graph", seq=2048, device=0, warmup=1, iters=3):
    buf = ctypes.create_string_buffer(1 << 20)
    rc = lib().kr_qwen_run(str(model_dir).encode(), mode.encode(), int(seq), int(device),
                           int(warmup), int(iters), buf, len(buf))
    return _decode(buf, rc)


def qwen_pp_run(model_dir, mode="pp", seq=2048, dev0=0, dev1=1, requests=2, warmup=1, iters=3):
    buf = ctypes.create_string_buffer(1 << 20)
    rc = lib().kr_qwen_pp_run(str(model_dir).encode(), mode.encode(), int(seq), int(dev0),
                              int(dev1), int(requests), int(warmup), int(iters), buf, len(buf))
    return _decode(buf, rc)


def qwen_tp_run(model_dir, mode="tp2", seq=2048, dev0=0, dev1=1, tiles=2, warmup=1, iters=3):
    """TP-MLP prefill.  mode tp{k} (NCCL AllReduce baseline) or tp{k}_split (relay)."""
    buf = ctypes.create_string_buffer(1 << 20)
    rc = lib().kr_qwen_tp_run(str(model_dir).encode(), mode.encode(), int(seq), int(dev0),
                              int(dev1), int(tiles), int(warmup), int(iters), buf, len(buf))
    return _decode(buf, rc)


def plan_run(schedule_json, devices="0,1", mode="direct", iters=3, warmup=1, out_json=None):
    """Run a reference-scheduler schedule.json through kr_plan_run; the library writes its
    result (or {"error": ...}) to `out_json`, which is read back here."""
    out = Path(out_json) if out_json else Path(tempfile.mkstemp(prefix="kr_plan_", suffix=".json")[1])
    rc = lib().kr_plan_run(str(schedule_json).encode(), int(iters), int(warmup),
                           str(devices).encode(), mode.encode(), str(out).encode())
    try:
        payload = json.loads(out.read_text(encoding="utf-8"))
    except Exception:
        payload = {"error": "no result", "rc": rc, "out": str(out)}
    payload["_rc"] = rc
    return payload


def qwen_profile_many(model_dir, cases, seq=2048, device=0):
    """Time a list of profile cases (each {"op": name, "k": slices}) against one loaded
    copy of the model through kr_qwen_profile_many; returns the decoded result JSON."""
    fd, path = tempfile.mkstemp(prefix="kr_profile_", suffix=".json")
    os.close(fd)
    Path(path).write_text(json.dumps({"cases": cases}), encoding="utf-8")
    buf = ctypes.create_string_buffer(4 << 20)
    try:
        rc = lib().kr_qwen_profile_many(str(model_dir).encode(), path.encode(), int(seq),
                                        int(device), buf, len(buf))
    finally:
        os.unlink(path)
    return _decode(buf, rc)
