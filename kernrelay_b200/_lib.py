"""ctypes binding of libkernrelay.so's B200 extension ABI (include/kernrelay_b200.h).

Everything here calls into the CUDA library; there is no Python or CPU fallback.
If the library is missing the import of the wrappers fails loudly.
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
_LIB = None

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_long = ctypes.c_long
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t
c_char_p = ctypes.c_char_p
c_u64 = ctypes.c_uint64
c_u32p = ctypes.POINTER(ctypes.c_uint32)


def lib_path() -> Path:
    env = os.environ.get("KERNRELAY_LIB")
    return Path(env) if env else _PKG / "libkernrelay.so"


# (name, restype, argtypes) of every exported symbol of include/kernrelay.h and
# include/kernrelay_b200.h; tests check the library exports exactly these.
SIGNATURES = [
    ("kr_version", c_char_p, []),
    ("kr_plan_run", c_int, [c_char_p, c_int, c_int, c_char_p, c_char_p, c_char_p]),
    ("kr_qwen_run", c_int, [c_char_p, c_char_p, c_int, c_int, c_int, c_int, c_char_p, c_size_t]),
    ("kr_qwen_pp_run", c_int, [c_char_p, c_char_p, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_char_p, c_size_t]),
    ("kr_qwen_tp_run", c_int, [c_char_p, c_char_p, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_char_p, c_size_t]),
    ("kr_qwen_profile_many", c_int, [c_char_p, c_char_p, c_int, c_int, c_char_p, c_size_t]),
    ("krb_last_error", c_char_p, []),
    ("krb_device_count", c_int, []),
    ("krb_synth_normal_host", c_int, [c_char_p, c_u64, ctypes.c_double, ctypes.c_double, c_u64,
                                      c_u64, c_void_p]),
    ("krb_gemm_bf16", c_int, [c_void_p, c_long, c_void_p, c_long, c_void_p, c_long, c_void_p,
                              c_int, c_int, c_int, c_int, c_void_p]),
    ("krb_gemm_f32out", c_int, [c_void_p, c_long, c_void_p, c_long, c_void_p, c_long, c_int, c_int,
                                c_int, c_int, c_void_p]),
    ("krb_gemm_silu_bf16", c_int, [c_void_p, c_long, c_void_p, c_long, c_void_p, c_long, c_int,
                                   c_int, c_int, c_int, c_void_p]),
    ("krb_gemm_qkv_rope_bf16", c_int, [c_void_p, c_long, c_void_p, c_long, c_void_p, c_long,
                                       c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_long,
                                       c_void_p]),
    ("krb_rmsnorm_bf16", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float,
                                 c_void_p]),
    ("krb_add_rmsnorm_bf16", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int, c_int, c_float, c_void_p]),
    ("krb_add_rmsnorm_res_f32", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                        c_int, c_float, c_void_p]),
    ("krb_embed_bf16", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                               c_void_p]),
    ("krb_qk_norm_rope_bf16", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_float, c_void_p]),
    ("krb_attention_prefill_bf16", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                           c_float, c_int, c_void_p, c_void_p]),
    ("krb_relay_down_single", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_int, c_float, c_int, c_void_p,
                                      c_void_p]),
    ("krb_relay_down_single_noalloc", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_int, c_int, c_int, c_int, c_float,
                                              c_int, c_void_p, c_void_p]),
    ("krb_relay_timeout_probe", c_int, [c_int, c_int, c_int, c_int, c_float, c_u32p]),
    ("krb_relay_plan", c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_char_p, c_size_t]),
    ("krb_plan_check", c_int, [c_char_p, c_char_p, c_size_t]),
    ("krb_engine_create", c_int, [c_char_p, c_char_p, c_int, c_int, c_int, c_int, c_int,
                                  ctypes.POINTER(c_void_p)]),
    ("krb_microdag_create", c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_char_p,
                                    c_u64, ctypes.POINTER(c_void_p)]),
    ("krb_engine_destroy", None, [c_void_p]),
    ("krb_engine_ipc_handle", c_int, [c_void_p, c_void_p, c_size_t]),
    ("krb_engine_open_peers", c_int, [c_void_p, c_void_p, c_size_t]),
    ("krb_nccl_unique_id", c_int, [c_void_p, c_size_t]),
    ("krb_engine_init_nccl", c_int, [c_void_p, c_void_p, c_size_t]),
    ("krb_engines_link", c_int, [ctypes.POINTER(c_void_p), c_int]),
    ("krb_engines_init_nccl", c_int, [ctypes.POINTER(c_void_p), c_int]),
    ("krb_engine_capture", c_int, [c_void_p]),
    ("krb_engine_run", c_int, [c_void_p]),
    ("krb_engine_run_host", c_int, [c_void_p, c_void_p, c_void_p]),
    ("krb_engine_sync", c_int, [c_void_p]),
    ("krb_engine_stream", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("krb_engine_status", c_int, [c_void_p, c_u32p]),
    ("krb_engine_stage_times", c_int, [c_void_p, c_char_p, c_size_t]),
    ("krb_engine_verify", c_int, [c_void_p, c_char_p, c_size_t]),
    ("krb_engine_last_logits", c_int, [c_void_p, c_void_p, c_int]),
    ("krb_engine_final_hidden", c_int, [c_void_p, c_void_p, c_size_t]),
    ("krb_engine_final_x", c_int, [c_void_p, c_void_p, c_size_t]),
    ("krb_engine_layer_dump", c_int, [c_void_p, c_int]),
    ("krb_engine_layer_hidden", c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    ("krb_engine_info", c_int, [c_void_p, c_char_p, c_size_t]),
    ("krb_engine_relay_trace", c_int, [c_void_p, c_void_p, c_size_t, ctypes.POINTER(c_size_t)]),
]


def lib():
    global _LIB
    if _LIB is None:
        p = lib_path()
        if not p.exists():
            raise FileNotFoundError(
                f"{p} is missing; build it with `python -m kernrelay_b200.build`")
        L = ctypes.CDLL(str(p))
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


class KrbError(RuntimeError):
    pass


def check(rc: int, what: str = ""):
    if rc != 0:
        msg = lib().krb_last_error().decode(errors="replace")
        raise KrbError(f"{what}: {msg}" if what else msg)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


# ---------------------------------------------------------------- tensor-level op wrappers
def gemm(A, B, bias=None, out=None, bn=0, stream=None):
    """C = A @ B.T (+bias): A [M,K], B [N,K] bf16 contiguous (row pitch may differ)."""
    import torch
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=A.device)
    check(lib().krb_gemm_bf16(_ptr(A), A.stride(0), _ptr(B), B.stride(0), _ptr(out), out.stride(0),
                              _ptr(bias), M, N, K, bn, _stream(stream)), "gemm")
    return out


def gemm_f32(A, B, out=None, bn=0, stream=None):
    """fp32 C = A @ B.T (unrounded)."""
    import torch
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    check(lib().krb_gemm_f32out(_ptr(A), A.stride(0), _ptr(B), B.stride(0), _ptr(out),
                                out.stride(0), M, N, K, bn, _stream(stream)), "gemm_f32")
    return out


def gemm_silu(A, Bgu, n_out, bn, out=None, stream=None):
    import torch
    M, K = A.shape
    if out is None:
        out = torch.empty((M, n_out), dtype=torch.bfloat16, device=A.device)
    check(lib().krb_gemm_silu_bf16(_ptr(A), A.stride(0), _ptr(Bgu), Bgu.stride(0), _ptr(out),
                                   out.stride(0), M, n_out, K, bn, _stream(stream)), "gemm_silu")
    return out


def interleave_gate_up(Wg, Wu, bn):
    """[I, K] gate and up rows -> the gate/up block interleave used by gemm_silu."""
    import torch
    I, K = Wg.shape
    half = bn // 2
    nblk = (I + half - 1) // half
    out = torch.zeros((nblk * bn, K), dtype=Wg.dtype, device=Wg.device)
    for b in range(nblk):
        lo, hi = b * half, min(I, (b + 1) * half)
        out[b * bn: b * bn + (hi - lo)] = Wg[lo:hi]
        out[b * bn + half: b * bn + half + (hi - lo)] = Wu[lo:hi]
    return out


def rmsnorm(x, gamma, eps, out=None, stream=None):
    import torch
    rows, H = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().krb_rmsnorm_bf16(_ptr(x), _ptr(gamma), _ptr(out), None, rows, H, eps,
                                 _stream(stream)), "rmsnorm")
    return out


def add_rmsnorm(a, b, gamma, eps, stream=None):
    import torch
    rows, H = a.shape
    y = torch.empty_like(a)
    s = torch.empty_like(a)
    check(lib().krb_add_rmsnorm_bf16(_ptr(a), _ptr(b), _ptr(gamma), _ptr(y), None, _ptr(s), rows,
                                     H, eps, _stream(stream)), "add_rmsnorm")
    return y, s


def add_rmsnorm_res(res, delta, gamma, eps, stream=None):
    """fp32 residual form: (y bf16, sum fp32) with sum = res + delta."""
    import torch
    rows, H = res.shape
    y = torch.empty((rows, H), dtype=torch.bfloat16, device=res.device)
    s = torch.empty_like(res)
    check(lib().krb_add_rmsnorm_res_f32(_ptr(res), _ptr(delta), _ptr(gamma), _ptr(y), _ptr(s), rows,
                                        H, eps, _stream(stream)), "add_rmsnorm_res")
    return y, s


def embed(ids, table, status=None, stream=None):
    import torch
    S = ids.shape[0]
    V, H = table.shape
    out = torch.empty((S, H), dtype=torch.bfloat16, device=table.device)
    check(lib().krb_embed_bf16(_ptr(ids), _ptr(table), _ptr(out), S, H, V, _ptr(status),
                               _stream(stream)), "embed")
    return out


def gemm_qkv_rope(A, B, HQ, HKV, D, cos, sin, bias=None, q_norm=None, k_norm=None, eps=1e-6,
                  vt=None, stream=None):
    """Fused QKV GEMM (+bias) with per-head QK-norm and RoPE in the epilogue; with `vt`
    (fp16 [HKV*D, ldvt >= M]) the v heads are also written transposed."""
    import torch
    M, K = A.shape
    N = (HQ + 2 * HKV) * D
    out = torch.empty((M, N), dtype=torch.bfloat16, device=A.device)
    check(lib().krb_gemm_qkv_rope_bf16(_ptr(A), A.stride(0), _ptr(B), B.stride(0), _ptr(out),
                                       out.stride(0), _ptr(bias), M, K, HQ, HKV, D, _ptr(cos),
                                       _ptr(sin), _ptr(q_norm), _ptr(k_norm), eps, _ptr(vt),
                                       vt.stride(0) if vt is not None else 0, _stream(stream)),
          "gemm_qkv_rope")
    return out


def qk_norm_rope(qkv, HQ, HKV, D, cos, sin, q_norm=None, k_norm=None, eps=1e-6, stream=None):
    S = qkv.shape[0]
    check(lib().krb_qk_norm_rope_bf16(_ptr(qkv), S, HQ, HKV, D, _ptr(cos), _ptr(sin), _ptr(q_norm),
                                      _ptr(k_norm), eps, _stream(stream)), "qk_norm_rope")
    return qkv


def attention(qkv, HQ, HKV, D, scale, impl=0, status=None, stream=None):
    """Causal GQA attention over the fused qkv buffer with the tcgen05 kernel (head_dim 64
    or 128); impl 0 and 2 both select it."""
    import torch
    S = qkv.shape[0]
    out = torch.empty((S, HQ * D), dtype=torch.bfloat16, device=qkv.device)
    check(lib().krb_attention_prefill_bf16(_ptr(qkv), _ptr(out), S, HQ, HKV, D, scale, impl,
                                           _ptr(status), _stream(stream)), "attention")
    return out


def relay_down_single(act, w_down, resid, gamma, tiles, eps, bn=0, status=None, stream=None):
    """resid fp32 [S,H] -> (sum fp32 [S,H], x bf16 [S,H])."""
    import torch
    S, K = act.shape
    H = w_down.shape[0]
    s = torch.empty((S, H), dtype=torch.float32, device=act.device)
    x = torch.empty((S, H), dtype=torch.bfloat16, device=act.device)
    check(lib().krb_relay_down_single(_ptr(act), _ptr(w_down), _ptr(resid), _ptr(gamma), _ptr(s),
                                      _ptr(x), S, H, K, tiles, eps, bn, _ptr(status),
                                      _stream(stream)), "relay_down_single")
    return s, x


def relay_down_single_noalloc(act, w_down, resid, gamma, tiles, eps, bn=0, status=None,
                              stream=None, out=None):
    """krb_relay_down_single_noalloc: same results as relay_down_single, no device
    allocation inside the library call (asynchronous on `stream`).  `out` may
    pass preallocated (sum fp32 [S,H], x bf16 [S,H])."""
    import torch
    S, K = act.shape
    H = w_down.shape[0]
    if out is None:
        out = (torch.empty((S, H), dtype=torch.float32, device=act.device),
               torch.empty((S, H), dtype=torch.bfloat16, device=act.device))
    s, x = out
    check(lib().krb_relay_down_single_noalloc(_ptr(act), _ptr(w_down), _ptr(resid), _ptr(gamma),
                                              _ptr(s), _ptr(x), S, H, K, tiles, eps, bn,
                                              _ptr(status), _stream(stream)),
          "relay_down_single_noalloc")
    return s, x


def synth_normal(name: str, seed: int, std: float, n: int, offset: int = 0, mean: float = 0.0):
    """bf16 bit pattern (uint16 numpy array) of a synthetic tensor (host, no GPU)."""
    import numpy as np
    out = np.empty(n, dtype=np.uint16)
    check(lib().krb_synth_normal_host(name.encode(), seed, std, mean, offset, n,
                                      out.ctypes.data_as(ctypes.c_void_p)), "synth")
    return out


def relay_timeout_probe(S, H, K, tiles, timeout_ms):
    """Status word of a relay whose only peer never runs (see kernrelay_b200.h)."""
    v = ctypes.c_uint32()
    check(lib().krb_relay_timeout_probe(S, H, K, tiles, timeout_ms, ctypes.byref(v)), "probe")
    return v.value


def relay_plan(S, H, tiles, k, rank, bn):
    buf = ctypes.create_string_buffer(1 << 16)
    rc = lib().krb_relay_plan(S, H, tiles, k, rank, bn, buf, len(buf))
    if rc != 0:
        raise KrbError(buf.value.decode(errors="replace"))
    return json.loads(buf.value.decode())


def plan_check(schedule_json):
    """Validate a schedule.json like kr_plan_run (no GPU needed); raises KrbError."""
    buf = ctypes.create_string_buffer(1 << 16)
    rc = lib().krb_plan_check(str(schedule_json).encode(), buf, len(buf))
    if rc != 0:
        raise KrbError(json.loads(buf.value.decode()).get("error", "plan check failed"))
    return json.loads(buf.value.decode())


# ---------------------------------------------------------------- per-rank engine
class Engine:
    """One rank of a prefill: owns its weights, activations and (split modes)
    its relay region.  For tp modes the ranks are wired with open_peers (split)
    or init_nccl (baseline) after all engines exist."""

    def __init__(self, model_dir, mode, seq, rank=0, world=1, device=0, tiles=4, _handle=None):
        h = _handle
        if h is None:
            h = c_void_p()
            check(lib().krb_engine_create(str(model_dir).encode(), mode.encode(), seq, rank, world,
                                          device, tiles, ctypes.byref(h)), "engine_create")
        self.h = h
        self.rank, self.world, self.device = rank, world, device

    @classmethod
    def microdag(cls, seq, hidden, intermediate, mode, rank=0, world=1, device=0, tiles=4,
                 seed=1234):
        """The isolated TP-MLP micro-DAG (krb_microdag_create): this rank's down GEMM over
        X_r, W_r, the reduction over the ranks and the Add+RMSNorm with R."""
        h = c_void_p()
        check(lib().krb_microdag_create(seq, hidden, intermediate, tiles, rank, world, device,
                                        mode.encode(), seed, ctypes.byref(h)), "microdag_create")
        return cls(None, mode, seq, rank=rank, world=world, device=device, tiles=tiles, _handle=h)

    def final_hidden(self):
        """fp32 [S, H] residual after the last layer (micro-DAG: h = R + sum of partials)."""
        import numpy as np
        info = self.info()
        n = info["seq"] * info["H"]
        out = np.empty(n, dtype=np.float32)
        check(lib().krb_engine_final_hidden(self.h, out.ctypes.data_as(c_void_p), n), "final_hidden")
        return out.reshape(info["seq"], info["H"])

    def final_x(self):
        """fp16 [S, H] final normed rows as fp32 numpy (micro-DAG: x = RMSNorm(h))."""
        import numpy as np
        info = self.info()
        n = info["seq"] * info["H"]
        out = np.empty(n, dtype=np.float16)
        check(lib().krb_engine_final_x(self.h, out.ctypes.data_as(c_void_p), n), "final_x")
        return out.astype(np.float32).reshape(info["seq"], info["H"])

    def close(self):
        if self.h:
            lib().krb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(lib().krb_engine_ipc_handle(self.h, buf, 64), "ipc_handle")
        return buf.raw

    def open_peers(self, handles: list[bytes]):
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(lib().krb_engine_open_peers(self.h, buf, len(blob)), "open_peers")

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().krb_nccl_unique_id(buf, 128), "nccl_unique_id")
        return buf.raw

    def init_nccl(self, uid: bytes):
        buf = ctypes.create_string_buffer(uid, len(uid))
        check(lib().krb_engine_init_nccl(self.h, buf, len(uid)), "init_nccl")

    @staticmethod
    def link(engines):
        arr = (c_void_p * len(engines))(*[e.h for e in engines])
        check(lib().krb_engines_link(arr, len(engines)), "engines_link")

    @staticmethod
    def init_nccl_all(engines):
        arr = (c_void_p * len(engines))(*[e.h for e in engines])
        check(lib().krb_engines_init_nccl(arr, len(engines)), "engines_init_nccl")

    def capture(self):
        check(lib().krb_engine_capture(self.h), "capture")

    def run(self):
        check(lib().krb_engine_run(self.h), "run")

    def run_host(self, ids_pinned, logits_pinned):
        check(lib().krb_engine_run_host(self.h, c_void_p(ids_pinned.data_ptr()),
                                        None if logits_pinned is None else
                                        c_void_p(logits_pinned.data_ptr())), "run_host")

    def sync(self):
        check(lib().krb_engine_sync(self.h), "sync")

    def stream_ptr(self) -> int:
        p = c_void_p()
        check(lib().krb_engine_stream(self.h, ctypes.byref(p)), "stream")
        return p.value or 0

    def status(self) -> int:
        v = ctypes.c_uint32()
        check(lib().krb_engine_status(self.h, ctypes.byref(v)), "status")
        return v.value

    def _json(self, fn, cap=1 << 16):
        buf = ctypes.create_string_buffer(cap)
        rc = fn(self.h, buf, cap)
        if rc != 0:
            raise KrbError(buf.value.decode(errors="replace"))
        return json.loads(buf.value.decode())

    def stage_times(self):
        return self._json(lib().krb_engine_stage_times)

    def verify(self):
        return self._json(lib().krb_engine_verify)

    def info(self):
        return self._json(lib().krb_engine_info)

    def last_logits(self):
        import numpy as np
        n = self.info()["V"]
        out = np.empty(n, dtype=np.float32)
        check(lib().krb_engine_last_logits(self.h, out.ctypes.data_as(c_void_p), n), "last_logits")
        return out

    TRACE_SLOTS = 48  # kTraceSlots in csrc/relay.cuh

    def relay_trace(self):
        """[grid, 48] globaltimer stamps of the last relay launch (KRB_RELAY_TRACE=1);
        slot meanings in csrc/relay.cuh (kTraceSlots)."""
        import numpy as np
        out = np.zeros(4096 * self.TRACE_SLOTS, dtype=np.uint64)
        n = c_size_t()
        check(lib().krb_engine_relay_trace(self.h, out.ctypes.data_as(c_void_p), out.size,
                                           ctypes.byref(n)), "relay_trace")
        return out[: n.value].reshape(-1, self.TRACE_SLOTS) if n.value else None

    def layer_dump(self, on=True):
        check(lib().krb_engine_layer_dump(self.h, 1 if on else 0), "layer_dump")

    def layer_hidden(self, layer):
        """fp32 residual stream after `layer` as numpy [S, H]."""
        import numpy as np
        info = self.info()
        n = info["seq"] * info["H"]
        out = np.empty(n, dtype=np.float32)
        check(lib().krb_engine_layer_hidden(self.h, layer, out.ctypes.data_as(c_void_p), n),
              "layer_hidden")
        return out.reshape(info["seq"], info["H"])
