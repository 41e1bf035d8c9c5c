"""ctypes wrapper of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, as the checker / the timed CPU restatement of
whisper.go's decoder. The product path never imports this module.
"""
from __future__ import annotations

import ctypes
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT / "whisper.go_b200"))
import wgdec  # noqa: E402  (descriptor structs shared with the product)

LIB_PATH = HERE / "liboracle.so"
_lib = None

fp = ctypes.POINTER(ctypes.c_float)
ip = ctypes.POINTER(ctypes.c_int32)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError("oracle/liboracle.so is missing: run __graft_entry__.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_row_bytes.restype = ctypes.c_int64
        L.or_row_bytes.argtypes = [ctypes.c_uint32, ctypes.c_int64]
        L.or_dequant.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int64, fp]
        L.or_dot_row.restype = ctypes.c_float
        L.or_dot_row.argtypes = [ctypes.c_uint32, ctypes.c_void_p, fp, ctypes.c_int]
        L.or_matmul.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, fp, ctypes.c_int, fp]
        L.or_set_inner_threads.argtypes = [ctypes.c_int]
        L.or_layernorm.argtypes = [fp, fp, fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.or_gelu_inplace.argtypes = [fp, ctypes.c_int64]
        L.or_fast_exp.restype = ctypes.c_float
        L.or_fast_exp.argtypes = [ctypes.c_float]
        L.or_softmax_fast.argtypes = [fp, ctypes.c_int]
        L.or_attention.argtypes = [fp, fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int64, ctypes.c_int, fp, fp]
        L.or_apply_penalty.argtypes = [fp, ctypes.c_int, ip, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        L.or_sample_greedy.restype = ctypes.c_int
        L.or_sample_greedy.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float]
        L.or_topk.restype = ctypes.c_int
        L.or_topk.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ip, fp]
        P = ctypes.POINTER(wgdec.WgModelDesc)
        L.or_decode.argtypes = [P, ctypes.POINTER(fp), ctypes.c_int, ctypes.c_int, ip, ctypes.c_int,
                                ctypes.POINTER(wgdec.WgDecodeParams), ip, ip, fp, ctypes.c_int]
        L.or_decode_trace.argtypes = [P, ctypes.POINTER(fp), ctypes.c_int, ctypes.c_int, ip, ctypes.c_int,
                                      ctypes.POINTER(wgdec.WgDecodeParams), ip, ip, fp, ctypes.c_int, fp, ip, ip,
                                      fp, ip, ip]
        L.or_sample_topp.restype = ctypes.c_int
        L.or_sample_topp.argtypes = [fp, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.or_uniform.restype = ctypes.c_float
        L.or_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32]
        L.or_topp_fallback.restype = ctypes.c_int
        L.or_topp_fallback.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float]
        L.or_teacher_forced.argtypes = [P, fp, ctypes.c_int, ip, ctypes.c_int, ip, ctypes.c_int, ctypes.c_int, fp]
        L.or_bench_steps.argtypes = [P, ctypes.c_int, ctypes.c_int, ip, ctypes.c_int,
                                     ctypes.POINTER(wgdec.WgDecodeParams), ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(fp)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError("oracle %s failed with status %d" % (what, rc))


def set_threads(n: int):
    lib().or_set_inner_threads(int(n))


def f32_to_f16(x: float) -> int:
    return int(lib().or_f32_to_f16(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().or_f16_to_f32(int(h)))


def dequant(qtype, raw: bytes, n: int) -> np.ndarray:
    qt = wgdec.QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    buf = np.frombuffer(bytes(raw), dtype=np.uint8).copy()
    out = np.empty(n, dtype=np.float32)
    _check(lib().or_dequant(qt, buf.ctypes.data, n, _f(out)), "dequant")
    return out


def dot_row(qtype, raw: bytes, f: np.ndarray) -> float:
    qt = wgdec.QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    buf = np.frombuffer(bytes(raw), dtype=np.uint8).copy()
    f = np.ascontiguousarray(f, dtype=np.float32)
    return float(lib().or_dot_row(qt, buf.ctypes.data, _f(f), f.size))


def matmul(qtype, raw, rows: int, cols: int, a: np.ndarray) -> np.ndarray:
    qt = wgdec.QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    buf = raw if isinstance(raw, np.ndarray) else np.frombuffer(bytes(raw), dtype=np.uint8).copy()
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty((a.shape[0], rows), dtype=np.float32)
    _check(lib().or_matmul(qt, buf.ctypes.data, rows, cols, _f(a), a.shape[0], _f(out)), "matmul")
    return out


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.empty_like(x2)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    lib().or_layernorm(_f(out), _f(x2), _f(w), _f(b), x2.shape[0], x2.shape[1], eps)
    return out.reshape(x.shape)


def gelu(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().or_gelu_inplace(_f(y), y.size)
    return y


def fast_exp(x: float) -> float:
    return float(lib().or_fast_exp(float(x)))


def softmax_fast(row: np.ndarray) -> np.ndarray:
    r = np.array(row, dtype=np.float32, copy=True)
    lib().or_softmax_fast(_f(r), r.size)
    return r


def attention(q, k, v, causal: bool):
    """q [H,Tq,hd], k/v [H,Tk,hd] -> out [H,Tq,hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    H, Tq, hd = q.shape
    Tk = k.shape[1]
    out = np.empty_like(q)
    sc = np.empty(Tq * Tk, dtype=np.float32)
    lib().or_attention(_f(q), _f(k), _f(v), H, Tq, Tk, hd, Tk * hd, int(causal), _f(out), _f(sc))
    return out


def apply_penalty(logits: np.ndarray, hist, penalty=2.0, window=128) -> np.ndarray:
    lg = np.array(logits, dtype=np.float32, copy=True)
    h = np.asarray(hist, dtype=np.int32)
    lib().or_apply_penalty(_f(lg), lg.size, h.ctypes.data_as(ip), h.size, penalty, window)
    return lg


def sample_greedy(logits, eot, temperature, suppress_nst=False, no_speech_thold=0.0) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().or_sample_greedy(_f(lg), lg.size, eot, temperature, int(suppress_nst), no_speech_thold))


def sample_topp(logits, temperature, u01, top_p=0.9) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().or_sample_topp(_f(lg), lg.size, temperature, top_p, u01))


def uniform(seed: int, u: int, t: int) -> float:
    """wg_uniform (include/wg_decoder.h): the seeded draw of the top-p sampler."""
    return float(lib().or_uniform(seed & 0xFFFFFFFFFFFFFFFF, u, t))


def topp_fallback(logits, chosen, temperature, logprob_thold) -> bool:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return bool(lib().or_topp_fallback(_f(lg), lg.size, int(chosen), temperature, logprob_thold))


def topk(logits, k, temperature):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    tok = np.zeros(k, dtype=np.int32)
    lp = np.zeros(k, dtype=np.float32)
    n = lib().or_topk(_f(lg), lg.size, k, temperature, tok.ctypes.data_as(ip), _f(lp))
    return tok[:n], lp[:n]


def _desc(model):
    d = model.desc if hasattr(model, "desc") else model
    if isinstance(d, ctypes._Pointer):
        return ctypes.cast(d, ctypes.POINTER(wgdec.WgModelDesc))
    return ctypes.cast(d, ctypes.POINTER(wgdec.WgModelDesc))


def decode(model, encs, params: "wgdec.DecoderParams", n_ctx: int, threads: int = 1):
    """Decode U utterances; returns (tokens [U, P+max_tokens], lens, scores)."""
    arrs = [np.ascontiguousarray(e, dtype=np.float32) for e in encs]
    ptrs = (fp * len(arrs))(*[_f(a) for a in arrs])
    pr = np.asarray(params.prompt, dtype=np.int32)
    mt = wgdec.max_tokens_for(params, n_ctx)
    stride = len(pr) + mt
    toks = np.zeros((len(arrs), stride), dtype=np.int32)
    lens = np.zeros(len(arrs), dtype=np.int32)
    scores = np.zeros(len(arrs), dtype=np.float32)
    cp = params.to_c()
    _check(lib().or_decode(_desc(model), ptrs, len(arrs), arrs[0].shape[0], pr.ctypes.data_as(ip), len(pr),
                           ctypes.byref(cp), toks.ctypes.data_as(ip), lens.ctypes.data_as(ip), _f(scores),
                           threads), "decode")
    return toks, lens, scores


def decode_trace(model, encs, params: "wgdec.DecoderParams", n_ctx: int, threads: int = 1):
    """decode() plus the per-step record: dict with tokens, lens, scores,
    margins [U, max_tokens] (the decision margin of each step: top-2 logit gap
    for greedy; for beams the smallest of every live row's 5th/6th logit gap
    and the gaps among the best B+1 candidates' normalised scores), steps [U],
    and for beam search beams_tokens [U, max_tokens, B, stride], beams_lens
    and beams_scores [U, max_tokens, B] (the beams after each step)."""
    arrs = [np.ascontiguousarray(e, dtype=np.float32) for e in encs]
    ptrs = (fp * len(arrs))(*[_f(a) for a in arrs])
    pr = np.asarray(params.prompt, dtype=np.int32)
    mt = wgdec.max_tokens_for(params, n_ctx)
    U, B, stride = len(arrs), max(1, int(params.beam_size)), len(pr) + mt
    toks = np.zeros((U, stride), dtype=np.int32)
    lens = np.zeros(U, dtype=np.int32)
    scores = np.zeros(U, dtype=np.float32)
    margins = np.zeros((U, max(mt, 1)), dtype=np.float32)
    btoks = np.zeros((U, max(mt, 1), B, stride), dtype=np.int32)
    blens = np.zeros((U, max(mt, 1), B), dtype=np.int32)
    bscores = np.zeros((U, max(mt, 1), B), dtype=np.float32)
    steps = np.zeros(U, dtype=np.int32)
    topp = np.zeros((U, max(mt, 1)), dtype=np.int32)
    cp = params.to_c()
    _check(lib().or_decode_trace(_desc(model), ptrs, U, arrs[0].shape[0], pr.ctypes.data_as(ip), len(pr),
                                 ctypes.byref(cp), toks.ctypes.data_as(ip), lens.ctypes.data_as(ip), _f(scores),
                                 threads, _f(margins), btoks.ctypes.data_as(ip), blens.ctypes.data_as(ip),
                                 _f(bscores), steps.ctypes.data_as(ip), topp.ctypes.data_as(ip)), "decode_trace")
    return dict(tokens=toks, lens=lens, scores=scores, margins=margins[:, :mt], steps=steps, topp=topp[:, :mt],
                beams_tokens=btoks[:, :mt], beams_lens=blens[:, :mt], beams_scores=bscores[:, :mt])


def teacher_forced(model, enc, prompt, forced, mode, n_vocab) -> np.ndarray:
    enc = np.ascontiguousarray(enc, dtype=np.float32)
    pr = np.asarray(prompt, dtype=np.int32)
    fo = np.asarray(forced, dtype=np.int32)
    out = np.empty((len(fo), n_vocab), dtype=np.float32)
    _check(lib().or_teacher_forced(_desc(model), _f(enc), enc.shape[0], pr.ctypes.data_as(ip), len(pr),
                                   fo.ctypes.data_as(ip), len(fo), mode, _f(out)), "teacher_forced")
    return out


def bench_steps(model, U, T, params: "wgdec.DecoderParams", n_steps: int, threads: int):
    pr = np.asarray(params.prompt, dtype=np.int32)
    cp = params.to_c()
    sec = ctypes.c_double()
    done = ctypes.c_int64()
    _check(lib().or_bench_steps(_desc(model), U, T, pr.ctypes.data_as(ip), len(pr), ctypes.byref(cp), n_steps,
                                threads, ctypes.byref(sec), ctypes.byref(done)), "bench_steps")
    return sec.value, done.value
