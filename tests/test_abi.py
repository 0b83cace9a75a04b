"""CPU: the C-ABI library loads without a GPU, exports exactly the symbols its headers
declare, and its error paths return the reference's conventions (rc + JSON error)."""
import json
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(kr_\w+|krb_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_exports_match_headers(krlib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(krlib.lib_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    exported = {n for n in exported if n.startswith(("kr_", "krb_"))}
    declared = _declared()
    assert declared == exported, (declared - exported, exported - declared)
    # the reference's six entry points are all there (include/kernrelay.h:11-69)
    for n in ("kr_version", "kr_plan_run", "kr_qwen_run", "kr_qwen_pp_run", "kr_qwen_tp_run",
              "kr_qwen_profile_many"):
        assert n in exported
    # and the ctypes table binds every one of them
    assert {n for n, _, _ in krlib.SIGNATURES} == declared


def test_version(krlib):
    from kernrelay_b200 import libapi
    assert libapi.version().startswith("KernRelay")


def test_plan_run_conventions(krlib, tmp_path):
    from kernrelay_b200 import libapi
    L = krlib.lib()
    assert L.kr_plan_run(None, 1, 1, None, None, b"x") == 2      # kr_api.cpp:27
    sched = tmp_path / "s.json"
    sched.write_text(json.dumps({"ranks": 1, "tasks": []}))
    r = libapi.plan_run(sched, devices="0", mode="direct", out_json=tmp_path / "o.json")
    assert r["_rc"] != 0 and "error" in r
    r = libapi.plan_run(sched, devices="0", mode="bogus", out_json=tmp_path / "o2.json")
    assert r["_rc"] != 0 and "unknown plan mode" in r["error"]


def test_run_errors_are_json_without_gpu(krlib, tmp_path):
    """Every runtime entry point reports failures as rc != 0 + {"error": ...}."""
    from kernrelay_b200 import libapi
    r = libapi.qwen_run(tmp_path / "missing", mode="serial", seq=64)
    assert r["_rc"] == 1 and "error" in r
    r = libapi.qwen_tp_run(tmp_path / "missing", mode="tp2_split", seq=64, dev0=0, dev1=0)
    assert r["_rc"] == 1 and "error" in r
    r = libapi.qwen_tp_run(tmp_path / "missing", mode="tp3", seq=64)
    assert r["_rc"] == 1 and "error" in r
    r = libapi.qwen_profile_many(tmp_path / "missing", [{"op": "rmsnorm", "k": 1}], seq=64)
    assert r["_rc"] == 1 and "error" in r
    r = libapi.qwen_pp_run(tmp_path / "missing", mode="pp", seq=64)
    assert r["_rc"] == 1 and "error" in r


@pytest.mark.parametrize("mode,dev0,dev1,requests,what", [
    ("pp", 0, 0, 2, "device2"),          # qwen_main.cpp:1995-1997
    ("pp", 0, 1, 0, "requests"),         # :1998-2000
    ("pp_serial", 0, 1, 9, "requests"),
    ("tp2", 0, 1, 2, "pp mode"),
])
def test_pp_run_rejects_bad_arguments(krlib, tmp_path, mode, dev0, dev1, requests, what):
    """kr_qwen_pp_run validates its arguments (as RunQwenPP does) before any device work."""
    from kernrelay_b200 import libapi
    r = libapi.qwen_pp_run(tmp_path, mode=mode, seq=64, dev0=dev0, dev1=dev1, requests=requests)
    assert r["_rc"] == 1 and what in r["error"]


def test_small_output_buffer_is_an_error(krlib, tmp_path):
    import ctypes
    buf = ctypes.create_string_buffer(8)
    rc = krlib.lib().kr_qwen_run(str(tmp_path).encode(), b"serial", 64, 0, 0, 1, buf, len(buf))
    assert rc == 1 and buf.value.startswith(b'{"err')


def test_device_count_never_fails(krlib):
    assert krlib.lib().krb_device_count() >= 0


@pytest.mark.parametrize("S,H,T,k,bn", [(2048, 3584, 4, 8, 256), (2048, 3584, 4, 2, 224),
                                        (512, 896, 4, 1, 256), (4096, 4096, 4, 8, 256),
                                        (2048, 2560, 2, 4, 128), (2048, 3584, 4, 1, 224)])
def test_relay_plan_counts(krlib, S, H, T, k, bn):
    """The relay GEMM's tile schedule covers every (128-row block, column) of the output
    exactly once; row tile t's counter target is the number of GEMM tiles whose rows lie in
    it (k = 1) or one forwarded signal per source (k > 1); a two-phase schedule runs at most
    one wave per phase.  Every rank owns a slice of every row tile, so every rank hears
    from every source."""
    plans = [krlib.relay_plan(S, H, T, k, r, bn) for r in range(k)]
    p0 = plans[0]
    R = S // T
    assert p0["R"] == R and p0["Rk"] * k == R
    cover = {}
    per_band = [0] * T
    cg = p0["cta_group"]
    for mb, nblk, n0, w in p0["tiles"]:
        assert w % (16 * cg) == 0 and 0 <= n0 < H and nblk == cg
        per_band[(mb * 128) // R] += 1
        for b in range(mb, mb + nblk):
            for c in range(n0, min(n0 + w, H), 16):
                cover[(b, c)] = cover.get((b, c), 0) + 1
    assert len(cover) == (S // 128) * len(range(0, H, 16)) and set(cover.values()) == {1}
    assert per_band == p0["band_tiles"] and p0["total"] == len(p0["tiles"])
    groups = p0["grid"] // cg
    if p0["p1"] < p0["total"]:
        assert p0["p1"] <= groups and p0["total"] - p0["p1"] <= groups and p0["bn2"] < bn
    for j in range(k):
        assert plans[j]["rs_expect"] == ([cg * n for n in p0["band_tiles"]] if k == 1 else [1] * T)
        assert plans[j]["ag_expect"] == (0 if k == 1 else 1)
    owners = {}
    for b, (tile, j0, j1) in enumerate(p0["blocks"]):
        assert tile == (b * 128) // R
        owners.setdefault(tile, set()).update(range(j0, j1 + 1))
    for t in range(T):
        assert owners[t] == set(range(k)), t


def test_relay_plan_two_phase_on_b200_7b(krlib, monkeypatch):
    """Qwen2.5-7B down_proj at S=2048, T=4, BN=224 on 148 SMs.  CTA pairs: 128 tiles of
    256x224 on 74 pairs (1.73 waves) become 74 phase-1 tiles plus 64 of width 192.  One-CTA
    tiles (KRB_GEMM_PAIR=0, read by a fresh library process): 256 tiles of 128x224 become
    148 plus 140 of width 176."""
    p = krlib.relay_plan(2048, 3584, 4, 2, 0, 224)
    if p["grid"] != 148:
        pytest.skip("not a 148-SM device")
    assert p["cta_group"] == 2
    assert p["p1"] == 74 and p["bn2"] == 192 and p["total"] == 138
    assert p["band_tiles"] == [32, 32, 10 + 26, 38]


def test_relay_plan_rejects_bad_shapes(krlib):
    with pytest.raises(krlib.KrbError):
        krlib.relay_plan(2048, 3584, 3, 2, 0, 256)     # 2048 % 3
    with pytest.raises(krlib.KrbError):
        krlib.relay_plan(2048, 3584, 32, 1, 0, 256)    # 64-row tiles < 128
    with pytest.raises(krlib.KrbError):
        krlib.relay_plan(2048, 3584, 4, 2, 2, 256)     # rank out of range


def test_relay_trace_summary_math():
    """kernrelay_b200.relay_trace turns per-CTA globaltimer stamps into per-tile phases and
    NVLink rates: direct pulls (k-1)*R*H*2 bytes per tile between 'partials arrived' and
    'norm done'."""
    import numpy as np
    from kernrelay_b200 import relay_trace
    tr = np.zeros((4, 48), dtype=np.uint64)
    base = 1_000_000
    tr[:, 0] = base
    tr[:, 1] = base + 100_000          # GEMM done at 100 us
    tr[:, 3] = base + 50_000           # tile 0 partials at 50 us
    tr[:, 6] = base + 60_000           # tile 0 norm done at 60 us
    s = relay_trace.summarise(tr, k=2, T=4, R=512, H=3584, kind="direct")
    assert s["gemm_done_us"] == 100.0
    t0 = s["tiles"][0]
    assert t0["partials_arrived_us"] == 50.0 and t0["norm_done_us"] == 60.0
    assert abs(t0["nvlink_gbs"] - 512 * 3584 * 2 / 10.0 / 1e3) < 1e-6
    assert "nvlink_gbs" not in s["tiles"][1]
