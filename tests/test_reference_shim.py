"""CPU: the reference's own, unmodified Python shim (python/kernrelay/libapi.py of a
KernRelay checkout) drives libkernrelay.so through KERNRELAY_LIB -- the drop-in claim
for its callers (scripts/run_qwen_tp.py, optimize.py, profile_model.py).

The checkout is taken from KRB_REFERENCE_CHECKOUT, else from a `reference` directory
beside this repository; without one the test is skipped.  Without a GPU every entry
point must come back through the shim's own convention: rc 1 and {"error": ...}.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _checkout():
    env = os.environ.get("KRB_REFERENCE_CHECKOUT")
    p = Path(env) if env else REPO.parent / "reference"
    return p if (p / "python" / "kernrelay" / "libapi.py").exists() else None


SCRIPT = r"""
import json, sys, tempfile
from pathlib import Path
from kernrelay import libapi as L   # the reference's shim, unmodified
td = Path(tempfile.mkdtemp())
out = {"lib_path": str(L.lib_path()), "version": L.version()}
out["qwen_run"] = L.qwen_run(td / "missing", mode="serial", seq=64, device=0)
out["qwen_tp_run"] = L.qwen_tp_run(td / "missing", mode="tp2_split", seq=64, dev0=0, dev1=1)
out["qwen_tp_run_bad_mode"] = L.qwen_tp_run(td / "missing", mode="tp3", seq=64)
out["qwen_pp_run"] = L.qwen_pp_run(td / "missing", mode="pp", seq=64, dev0=0, dev1=1)
out["plan_run"] = L.plan_run(td / "missing.json", devices="0", out_json=td / "o.json")
out["qwen_profile_many"] = L.qwen_profile_many(td / "missing", [{"op": "rmsnorm", "k": 1}],
                                                seq=64, device=0)
print(json.dumps(out))
"""


def test_reference_libapi_drives_this_library(krlib, tmp_path):
    ref = _checkout()
    if ref is None:
        pytest.skip("no KernRelay checkout (set KRB_REFERENCE_CHECKOUT)")
    env = dict(os.environ, PYTHONPATH=str(ref / "python"), KERNRELAY_LIB=str(krlib.lib_path()),
               CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, "-c", SCRIPT], cwd=tmp_path, env=env,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    out = json.loads(p.stdout.strip().splitlines()[-1])
    assert Path(out["lib_path"]).resolve() == krlib.lib_path().resolve()
    assert out["version"].startswith("KernRelay 0.3 (libkernrelay")
    for name in ("qwen_run", "qwen_tp_run", "qwen_tp_run_bad_mode", "qwen_pp_run", "plan_run",
                 "qwen_profile_many"):
        r = out[name]
        assert r["_rc"] == 1, (name, r)
        assert isinstance(r.get("error"), str) and r["error"], (name, r)
    assert "tp" in out["qwen_tp_run_bad_mode"]["error"]
