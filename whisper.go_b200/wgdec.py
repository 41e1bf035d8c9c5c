"""Host-side mirror of whisper.go's decoder plugin interface over the C ABI.

`WhisperDecoder.decode(encoder_out, params, ctx)` mirrors
    model.Decoder.Decode(ctx, encoderOut ml.Tensor, params DecoderParams)
        ([]Segment, error)                     (internal/model/interfaces.go:22-25)
with `DecoderParams`, `Segment` and `TokenData` mirroring interfaces.go:47-90
and the error convention of internal/model/decoder.go (errors prefixed
"model: decode: ...", cancellation surfaced as an error whose cause is
`Canceled`, like errors.Is(err, context.Canceled)).

Everything below the C ABI (include/wg_decoder.h) runs on the GPU; this
module only marshals arguments. There is no CPU fallback: if libwgdec.so is
missing the import of the library raises.
"""
from __future__ import annotations

import ctypes
import dataclasses
import pathlib
import threading
from typing import List, Optional, Sequence

import numpy as np

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
LIB_PATH = PKG / "libwgdec.so"
GEN_PATH = PKG / "libwggen.so"

QTYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8}
QTYPE_NAMES = {v: k for k, v in QTYPES.items()}
MODE_REF_COMPAT = 0
MODE_CORRECT = 1

WG_OK = 0
STATUS = {0: "ok", 1: "invalid", 2: "cuda", 3: "oom", 4: "unsupported", 5: "cancelled", 6: "timeout",
          7: "injected", 8: "no_device", 9: "device_flag"}
KCLASS = {"gemv": 0, "self_attn": 1, "cross_attn": 2, "logits": 3, "precompute": 4, "step": 5,
          "qkv": 10, "self_out": 11, "cross_q": 12, "cross_out": 13, "mlp0": 14, "mlp2": 15}

c_float_p = ctypes.POINTER(ctypes.c_float)
c_int32_p = ctypes.POINTER(ctypes.c_int32)


class WgMatrix(ctypes.Structure):
    _fields_ = [("qtype", ctypes.c_uint32), ("rows", ctypes.c_int32), ("cols", ctypes.c_int32),
                ("data", ctypes.c_void_p)]


class WgLayerDesc(ctypes.Structure):
    _fields_ = [
        ("self_ln_w", c_float_p), ("self_ln_b", c_float_p),
        ("self_q", WgMatrix), ("self_q_b", c_float_p),
        ("self_k", WgMatrix),
        ("self_v", WgMatrix), ("self_v_b", c_float_p),
        ("self_o", WgMatrix), ("self_o_b", c_float_p),
        ("cross_ln_w", c_float_p), ("cross_ln_b", c_float_p),
        ("cross_q", WgMatrix), ("cross_q_b", c_float_p),
        ("cross_k", WgMatrix),
        ("cross_v", WgMatrix), ("cross_v_b", c_float_p),
        ("cross_o", WgMatrix), ("cross_o_b", c_float_p),
        ("mlp_ln_w", c_float_p), ("mlp_ln_b", c_float_p),
        ("mlp0", WgMatrix), ("mlp0_b", c_float_p),
        ("mlp2", WgMatrix), ("mlp2_b", c_float_p),
    ]


class WgModelDesc(ctypes.Structure):
    _fields_ = [
        ("n_vocab", ctypes.c_int32), ("n_state", ctypes.c_int32), ("n_head", ctypes.c_int32),
        ("n_layer", ctypes.c_int32), ("n_text_ctx", ctypes.c_int32), ("eot", ctypes.c_int32),
        ("token_embedding", WgMatrix),
        ("positional_embedding", c_float_p),
        ("ln_w", c_float_p), ("ln_b", c_float_p),
        ("layers", ctypes.POINTER(WgLayerDesc)),
    ]


class WgDecodeParams(ctypes.Structure):
    _fields_ = [
        ("beam_size", ctypes.c_int32), ("temperature", ctypes.c_float), ("attempt", ctypes.c_int32),
        ("logprob_thold", ctypes.c_float), ("no_speech_thold", ctypes.c_float),
        ("no_fallback", ctypes.c_int32), ("max_tokens", ctypes.c_int32), ("suppress_nst", ctypes.c_int32),
        ("mode", ctypes.c_int32), ("suppress_eot", ctypes.c_int32), ("seed", ctypes.c_uint64),
    ]


_lib = None
_gen = None
_lock = threading.Lock()


def _declare(lib):
    P = ctypes.c_void_p
    sig = {
        "wg_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
        "wg_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
        "wg_kernel_launch_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int64)]),
        "wg_model_create": (ctypes.c_int, [ctypes.POINTER(WgModelDesc), ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                           ctypes.POINTER(P)]),
        "wg_model_create_from_gguf": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                                     ctypes.POINTER(P)]),
        "wg_model_destroy": (ctypes.c_int, [P]),
        "wg_model_weight_bytes": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "wg_model_set_eot": (ctypes.c_int, [P, ctypes.c_int]),
        "wg_model_info": (ctypes.c_int, [P] + [ctypes.POINTER(ctypes.c_int)] * 5),
        "wg_job_create": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, c_int32_p, ctypes.c_int,
                                         ctypes.POINTER(WgDecodeParams), ctypes.POINTER(P)]),
        "wg_job_upload_encoder": (ctypes.c_int, [P, ctypes.POINTER(c_float_p)]),
        "wg_job_upload_encoder_device": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
        "wg_job_utterance_device": (ctypes.c_int, [P, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
        "wg_job_start": (ctypes.c_int, [P]),
        "wg_job_step": (ctypes.c_int, [P, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
        "wg_job_result": (ctypes.c_int, [P, c_int32_p, c_int32_p, c_float_p]),
        "wg_job_beams": (ctypes.c_int, [P, c_int32_p, c_int32_p, c_float_p]),
        "wg_job_cancel": (ctypes.c_int, [P]),
        "wg_job_timer": (ctypes.c_int, [P, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]),
        "wg_job_destroy": (ctypes.c_int, [P]),
        "wg_job_uses_step_kernel": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int)]),
        "wg_job_stats": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                        ctypes.POINTER(ctypes.c_int)]),
        "wg_decode": (ctypes.c_int, [P, ctypes.POINTER(c_float_p), ctypes.c_int, ctypes.c_int, c_int32_p,
                                     ctypes.c_int, ctypes.POINTER(WgDecodeParams), c_int32_p, c_int32_p, c_float_p]),
        "wg_teacher_forced_logits": (ctypes.c_int, [P, ctypes.POINTER(c_float_p), ctypes.c_int, ctypes.c_int,
                                                    c_int32_p, ctypes.c_int, c_int32_p, ctypes.c_int, ctypes.c_int,
                                                    c_float_p]),
        "wg_batcher_create": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(P)]),
        "wg_batcher_decode": (ctypes.c_int, [P, c_float_p, ctypes.c_int, c_int32_p, ctypes.c_int,
                                             ctypes.POINTER(WgDecodeParams), ctypes.POINTER(ctypes.c_int), c_int32_p,
                                             ctypes.c_int, c_int32_p, c_float_p]),
        "wg_batcher_stats": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
        "wg_batcher_destroy": (ctypes.c_int, [P]),
        "wg_dequant_test": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int64, c_float_p]),
        "wg_matmul_test": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, c_float_p,
                                          ctypes.c_int, c_float_p, ctypes.c_int]),
        "wg_sample_test": (ctypes.c_int, [c_float_p, ctypes.c_int, ctypes.c_int, c_int32_p, ctypes.c_int,
                                          ctypes.c_int, ctypes.POINTER(WgDecodeParams), ctypes.c_int, c_int32_p,
                                          c_float_p]),
        "wg_job_time_kernel": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                              ctypes.POINTER(ctypes.c_double)]),
        "wg_model_matmul_noalloc": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                   ctypes.c_void_p, ctypes.c_int]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def lib():
    """The CUDA library. Raises if it was not built (no CPU fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError("libwgdec.so is missing: run __graft_entry__.build() (no CPU fallback)")
            _lib = _declare(ctypes.CDLL(str(LIB_PATH)))
        return _lib


def gen():
    global _gen
    with _lock:
        if _gen is None:
            if not GEN_PATH.exists():
                raise RuntimeError("libwggen.so is missing: run __graft_entry__.build()")
            g = ctypes.CDLL(str(GEN_PATH))
            g.wg_gen_model_create.restype = ctypes.POINTER(WgModelDesc)
            g.wg_gen_model_create.argtypes = [ctypes.c_int] * 5 + [ctypes.c_uint32, ctypes.c_uint64]
            g.wg_gen_model_free.argtypes = [ctypes.POINTER(WgModelDesc)]
            g.wg_gen_encoder.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_float_p]
            g.wg_gen_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_float, c_float_p]
            g.wg_gen_quantize.restype = ctypes.c_int64
            g.wg_gen_quantize.argtypes = [ctypes.c_uint32, c_float_p, ctypes.c_int64, ctypes.c_void_p]
            g.wg_gen_quantize_matrix.argtypes = [ctypes.c_uint32, c_float_p, ctypes.c_int64, ctypes.c_int64,
                                                 ctypes.c_void_p]
            g.wg_gen_row_bytes.restype = ctypes.c_int64
            g.wg_gen_row_bytes.argtypes = [ctypes.c_uint32, ctypes.c_int64]
            g.wg_gen_f32_to_f16.restype = ctypes.c_uint16
            g.wg_gen_f32_to_f16.argtypes = [ctypes.c_float]
            _gen = g
        return _gen


class DecodeError(RuntimeError):
    """A failed Decode; `status` is the C ABI status code."""

    def __init__(self, msg: str, status: int = 1):
        super().__init__(msg)
        self.status = status


class Canceled(Exception):
    """Mirror of context.Canceled."""

    def __str__(self):
        return "context canceled"


class Context:
    """Minimal mirror of context.Context: cancel() and err()."""

    def __init__(self):
        self._canceled = threading.Event()

    def cancel(self):
        self._canceled.set()

    def err(self):
        return Canceled() if self._canceled.is_set() else None


def is_canceled(err: BaseException) -> bool:
    """errors.Is(err, context.Canceled)."""
    e = err
    while e is not None:
        if isinstance(e, Canceled):
            return True
        e = e.__cause__
    return False


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().wg_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = ""):
    if rc != WG_OK:
        msg = last_error()
        if not msg.startswith("model:"):
            msg = "model: decode: %s%s" % (what + ": " if what else "", msg)
        err = DecodeError(msg, rc)
        if rc == 5:
            raise err from Canceled()
        raise err


def device_count() -> int:
    n = ctypes.c_int(0)
    lib().wg_device_count(ctypes.byref(n))
    return n.value


def kernel_launch_count() -> int:
    n = ctypes.c_int64(0)
    lib().wg_kernel_launch_count(ctypes.byref(n))
    return n.value


# ---- parameters and results (internal/model/interfaces.go:47-90) ------------
@dataclasses.dataclass
class DecoderParams:
    prompt: Sequence[int] = ()
    beam_size: int = 1
    best_of: int = 0            # never read by the reference decoder
    temperature: float = 0.0
    temperature_inc: float = 0.0  # never read by the reference decoder
    entropy_thold: float = 0.0    # never read
    logprob_thold: float = 0.0
    no_speech_thold: float = 0.0
    no_fallback: bool = False
    max_tokens: int = 0
    suppress_nst: bool = False
    suppress_regex: str = ""      # never read
    dtw_enabled: bool = False     # never read
    # build switches (not in the reference)
    mode: int = MODE_CORRECT
    suppress_eot: bool = False
    attempt: int = 0
    seed: int = 0                 # top-p draws: wg_uniform(seed, utterance, step)

    def to_c(self) -> WgDecodeParams:
        return WgDecodeParams(beam_size=int(self.beam_size), temperature=float(self.temperature),
                              attempt=int(self.attempt), logprob_thold=float(self.logprob_thold),
                              no_speech_thold=float(self.no_speech_thold), no_fallback=int(bool(self.no_fallback)),
                              max_tokens=int(self.max_tokens), suppress_nst=int(bool(self.suppress_nst)),
                              mode=int(self.mode), suppress_eot=int(bool(self.suppress_eot)),
                              seed=int(self.seed) & 0xFFFFFFFFFFFFFFFF)


def max_tokens_for(params: DecoderParams, n_text_ctx: int) -> int:
    """internal/model/decoder.go:421-430."""
    mt = params.max_tokens
    if mt <= 0:
        mt = n_text_ctx
    mt = min(mt, n_text_ctx - len(params.prompt))
    return max(mt, 0)


@dataclasses.dataclass
class TokenData:
    id: int
    text: str = ""
    p: float = 0.0
    plog: float = 0.0
    pt: float = 0.0
    ptsum: float = 0.0
    t0: int = 0
    t1: int = 0
    tdtw: int = 0


@dataclasses.dataclass
class Segment:
    start_ms: int = 0
    end_ms: int = 0
    text: str = ""
    tokens: List[TokenData] = dataclasses.field(default_factory=list)
    speaker: int = 0


def collapse_repeated_substrings(s: str, max_unit_len: int = 6, min_repeats: int = 3) -> str:
    """internal/model/decoder.go:1188-1230 (collapseRepeatedSubstrings), on UTF-8 bytes."""
    if not s or max_unit_len <= 0 or min_repeats <= 1:
        return s
    b = s.encode("utf-8")
    n, i, out = len(b), 0, bytearray()
    while i < n:
        collapsed = False
        for ln in range(1, min(max_unit_len, n - i) + 1):
            unit = b[i:i + ln]
            cnt, j = 1, i + ln
            while j + ln <= n and b[j:j + ln] == unit:
                cnt += 1
                j += ln
                if cnt >= min_repeats:
                    break
            if cnt >= min_repeats:
                out += unit
                i += ln * cnt
                collapsed = True
                break
        if not collapsed:
            out.append(b[i])
            i += 1
    return out.decode("utf-8", errors="replace")


def compression_ratio(text: str) -> float:
    """internal/model/decoder.go:1170-1183 (compressionRatio): byte length over
    gzip length at the default level (6). Go's compress/flate and zlib are
    different deflate implementations, so the compressed length can differ by
    a few bytes from the reference's."""
    import gzip
    if not text:
        return 0.0
    raw = text.encode("utf-8")
    comp = len(gzip.compress(raw, compresslevel=6, mtime=0))
    return float(np.float32(len(raw)) / np.float32(comp)) if comp else float(len(raw))


def tokens_to_segments(tokens: Sequence[int], prompt: Sequence[int], vocab=None) -> List[Segment]:
    """internal/model/decoder.go:1415-1459: one segment of the non-prompt
    tokens; with a vocabulary (decode_token / decode, like vocab.Vocabulary)
    consecutive tokens with the same non-empty text are collapsed and the
    segment text is the decoded rest with repeated substrings collapsed."""
    if len(tokens) < len(prompt):
        return []
    rest = [int(t) for t in tokens[len(prompt):]]
    if not rest:
        return []
    seg = Segment()
    last, kept = "", []
    for t in rest:
        text = vocab.decode_token(t) if vocab is not None else ""
        if text and text == last:
            continue
        last = text
        seg.tokens.append(TokenData(id=t, text=text))
        kept.append(t)
    if vocab is not None:
        seg.text = collapse_repeated_substrings(vocab.decode(kept), 6, 3)
    return [seg]


# ---- model descriptors ----------------------------------------------------------
class SyntheticModel:
    """Seeded synthetic decoder (whisper.go_b200/gen/wg_gen.c) in one qtype."""

    def __init__(self, n_vocab, d, n_head, n_layer, n_ctx=448, qtype="Q8_0", seed=1234):
        qt = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
        self.ptr = gen().wg_gen_model_create(n_vocab, d, n_head, n_layer, n_ctx, qt, seed)
        if not self.ptr:
            raise MemoryError("synthetic model generation failed")
        self.n_vocab, self.d, self.n_head, self.n_layer, self.n_ctx = n_vocab, d, n_head, n_layer, n_ctx
        self.qtype, self.seed = qt, seed

    @property
    def desc(self):
        return self.ptr

    def encoder_output(self, u: int, T: int = 1500, seed: Optional[int] = None) -> np.ndarray:
        out = np.empty((T, self.d), dtype=np.float32)
        gen().wg_gen_encoder(self.seed if seed is None else seed, u, T, self.d,
                             out.ctypes.data_as(c_float_p))
        return out

    def close(self):
        if self.ptr:
            gen().wg_gen_model_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ArrayModel:
    """A decoder descriptor built from numpy arrays (dense or raw GGUF bytes).

    weights: dict with keys token_embedding, positional_embedding, ln_w, ln_b
    and a list `layers` of dicts with the wg_layer_desc field names; matrices
    are (qtype, rows, cols, bytes-or-float32-array).
    """

    def __init__(self, n_vocab, d, n_head, n_layer, n_ctx, weights, eot=50256):
        self._keep = []
        self.n_vocab, self.d, self.n_head, self.n_layer, self.n_ctx = n_vocab, d, n_head, n_layer, n_ctx

        def vec(a):
            a = np.ascontiguousarray(a, dtype=np.float32)
            self._keep.append(a)
            return a.ctypes.data_as(c_float_p)

        def mat(spec):
            qt, rows, cols, data = spec
            qt = QTYPES[qt] if isinstance(qt, str) else int(qt)
            if isinstance(data, np.ndarray) and data.dtype == np.float32:
                buf = np.ascontiguousarray(data)
            else:
                buf = np.frombuffer(bytes(data), dtype=np.uint8).copy()
            self._keep.append(buf)
            return WgMatrix(qt, rows, cols, buf.ctypes.data)

        self._layers = (WgLayerDesc * n_layer)()
        for i, L in enumerate(weights["layers"]):
            ld = self._layers[i]
            for name, _ in WgLayerDesc._fields_:
                v = L[name]
                setattr(ld, name, mat(v) if isinstance(v, tuple) else vec(v))
        self._desc = WgModelDesc(n_vocab=n_vocab, n_state=d, n_head=n_head, n_layer=n_layer, n_text_ctx=n_ctx,
                                 eot=eot, token_embedding=mat(weights["token_embedding"]),
                                 positional_embedding=vec(weights["positional_embedding"]),
                                 ln_w=vec(weights["ln_w"]), ln_b=vec(weights["ln_b"]),
                                 layers=ctypes.cast(self._layers, ctypes.POINTER(WgLayerDesc)))

    @property
    def desc(self):
        return ctypes.pointer(self._desc)


def _desc_ptr(model_desc):
    d = model_desc.desc if hasattr(model_desc, "desc") else model_desc
    if isinstance(d, ctypes._Pointer):
        return d
    return ctypes.cast(d, ctypes.POINTER(WgModelDesc))


def _enc_array(encs: Sequence[np.ndarray]):
    arrs = [np.ascontiguousarray(e, dtype=np.float32) for e in encs]
    ptrs = (c_float_p * len(arrs))(*[a.ctypes.data_as(c_float_p) for a in arrs])
    return arrs, ptrs


# ---- the decoder ----------------------------------------------------------------
class WhisperDecoder:
    """GPU replacement of internal/model/decoder.go's WhisperDecoder."""

    def __init__(self, model_desc, devices: Optional[Sequence[int]] = None):
        self._src = model_desc
        d = _desc_ptr(model_desc).contents
        self.n_vocab, self.n_state, self.n_head = d.n_vocab, d.n_state, d.n_head
        self.n_layer, self.n_text_ctx, self.eot = d.n_layer, d.n_text_ctx, d.eot
        h = ctypes.c_void_p()
        devs = None
        nd = 0
        if devices:
            devs = (ctypes.c_int * len(devices))(*devices)
            nd = len(devices)
        check(lib().wg_model_create(_desc_ptr(model_desc), devs, nd, ctypes.byref(h)), "model create")
        self.h = h
        self.vocab = None

    @classmethod
    def from_gguf(cls, path, devices: Optional[Sequence[int]] = None) -> "WhisperDecoder":
        """NewDecoder on a GGUF model file (wg_model_create_from_gguf)."""
        self = cls.__new__(cls)
        self._src = None
        h = ctypes.c_void_p()
        devs = (ctypes.c_int * len(devices))(*devices) if devices else None
        check(lib().wg_model_create_from_gguf(str(path).encode(), devs, len(devices) if devices else 0,
                                              ctypes.byref(h)), "model create")
        self.h = h
        self.vocab = None
        self.eot = 50256
        vals = [ctypes.c_int() for _ in range(5)]
        check(lib().wg_model_info(h, *[ctypes.byref(v) for v in vals]))
        self.n_vocab, self.n_state, self.n_head, self.n_layer, self.n_text_ctx = [v.value for v in vals]
        return self

    def weight_bytes(self) -> int:
        n = ctypes.c_int64()
        check(lib().wg_model_weight_bytes(self.h, ctypes.byref(n)))
        return n.value

    def close(self):
        if getattr(self, "h", None):
            lib().wg_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_vocabulary(self, vocab):
        """SetVocabulary (decoder.go:85-95): token text for the segments, the
        compression-ratio retry, and the vocabulary's EOT id (vocab.eot >= 0)."""
        self.vocab = vocab
        eot = getattr(vocab, "eot", -1) if vocab is not None else -1
        if eot is not None and eot >= 0:
            check(lib().wg_model_set_eot(self.h, int(eot)), "set vocabulary")
            self.eot = int(eot)

    # Decode (interfaces.go:22-25)
    def decode(self, encoder_out: np.ndarray, params: DecoderParams, ctx: Optional[Context] = None) -> List[Segment]:
        return self.decode_batch([encoder_out], params, ctx)[0]

    ATTEMPTS = 3  # decoder.go:415, :534

    def decode_batch(self, encoder_outs: Sequence[np.ndarray], params: DecoderParams,
                     ctx: Optional[Context] = None) -> List[List[Segment]]:
        """Decode of every utterance, with the reference's retry schedule when
        a vocabulary is set (decoder.go:433-515 greedy, :536-716 beam): an
        utterance whose decoded text compresses by more than 2.4 is decoded
        again at temperature + 0.2 * attempt, up to 3 attempts, unless
        NoFallback. Retries of several utterances run as one batch."""
        vocab = getattr(self, "vocab", None)
        U, P = len(encoder_outs), len(params.prompt)
        final = [None] * U
        pending = list(range(U))
        for attempt in range(self.ATTEMPTS if vocab is not None else 1):
            p = dataclasses.replace(params, attempt=attempt) if vocab is not None else params
            toks, lens, _ = self.decode_tokens([encoder_outs[u] for u in pending], p, ctx)
            retry = []
            for k, u in enumerate(pending):
                final[u] = toks[k, :lens[k]]
                gen = [int(t) for t in final[u][P:]]
                if vocab is None or not gen:
                    continue
                text = vocab.decode(gen)
                if text and compression_ratio(text) > 2.4 and attempt < self.ATTEMPTS - 1 and not params.no_fallback:
                    retry.append(u)
            pending = retry
            if not pending:
                break
        return [tokens_to_segments(final[u], params.prompt, vocab) for u in range(U)]

    def decode_tokens(self, encoder_outs, params: DecoderParams, ctx: Optional[Context] = None, stream: int = 0):
        """Tokens [U, P+max_tokens], lens [U], scores [U]. Encoder outputs are
        host arrays, or device tensors (objects with data_ptr() and is_cuda,
        fp32 contiguous [T, d], on the utterance's device) handed over on the
        device after `stream` (cudaStream_t value of their producer)."""
        for e in encoder_outs:
            if e.ndim != 2 or e.shape[1] != self.n_state:
                raise DecodeError("model: decoder: encoder output must be [T, %d], got %s" % (self.n_state,
                                                                                           list(e.shape)))
        if ctx is not None and ctx.err() is not None:
            raise DecodeError("model: decode: cancelled: context canceled", 5) from ctx.err()
        on_device = all(getattr(e, "is_cuda", False) for e in encoder_outs)
        job = Job(self, len(encoder_outs), encoder_outs[0].shape[0], params)
        try:
            if on_device:
                job.upload_device([e.data_ptr() for e in encoder_outs], stream)
            else:
                job.upload(encoder_outs)
            job.start()
            done = False
            while not done:
                if ctx is not None and ctx.err() is not None:
                    job.cancel()
                done = job.step(16)
            return job.result()
        finally:
            job.close()

    def teacher_forced_logits(self, encoder_outs, prompt: Sequence[int], forced, mode: int = MODE_CORRECT
                              ) -> np.ndarray:
        """Logits [n_forced, U, V] along forced token sequences (forced: [U, n] or [n])."""
        if isinstance(encoder_outs, np.ndarray) and encoder_outs.ndim == 2:
            encoder_outs = [encoder_outs]
        arrs, ptrs = _enc_array(encoder_outs)
        U = len(arrs)
        pr = np.asarray(prompt, dtype=np.int32)
        fo = np.ascontiguousarray(np.asarray(forced, dtype=np.int32).reshape(U, -1))
        n = fo.shape[1]
        out = np.empty((n, U, self.n_vocab), dtype=np.float32)
        check(lib().wg_teacher_forced_logits(self.h, ptrs, U, arrs[0].shape[0], pr.ctypes.data_as(c_int32_p),
                                             len(pr), fo.ctypes.data_as(c_int32_p), n, mode,
                                             out.ctypes.data_as(c_float_p)), "teacher forcing")
        return out


class Batcher:
    """Pipeline batching (wg_batcher_*): decode() from many threads at once;
    compatible calls within `window_us` share one GPU job (ctypes releases
    the GIL for the blocking call, so the threads wait in parallel)."""

    def __init__(self, dec: WhisperDecoder, max_utterances: int = 64, window_us: int = 2000):
        self.dec = dec
        h = ctypes.c_void_p()
        check(lib().wg_batcher_create(dec.h, max_utterances, window_us, ctypes.byref(h)), "batcher")
        self.h = h

    def decode_tokens(self, encoder_out: np.ndarray, params: DecoderParams, ctx: Optional[Context] = None):
        """(tokens, score) of one utterance, prompt included."""
        enc = np.ascontiguousarray(encoder_out, dtype=np.float32)
        pr = np.asarray(params.prompt, dtype=np.int32)
        cap = len(pr) + max_tokens_for(params, self.dec.n_text_ctx)
        toks = np.zeros(max(cap, 1), dtype=np.int32)
        n = ctypes.c_int32(0)
        sc = ctypes.c_float(0)
        cp = params.to_c()
        flag = ctypes.c_int(0)
        watcher = None
        if ctx is not None:  # ctx.Done() -> the request's cancel flag
            def watch():
                ctx._canceled.wait()
                flag.value = 1
            watcher = threading.Thread(target=watch, daemon=True)
            watcher.start()
        check(lib().wg_batcher_decode(self.h, enc.ctypes.data_as(c_float_p), enc.shape[0], pr.ctypes.data_as(c_int32_p),
                                      len(pr), ctypes.byref(cp), ctypes.byref(flag), toks.ctypes.data_as(c_int32_p),
                                      len(toks), ctypes.byref(n), ctypes.byref(sc)), "batcher")
        return toks[:n.value], sc.value

    def decode(self, encoder_out: np.ndarray, params: DecoderParams, ctx: Optional[Context] = None) -> List[Segment]:
        toks, _ = self.decode_tokens(encoder_out, params, ctx)
        return tokens_to_segments(toks, params.prompt, getattr(self.dec, "vocab", None))

    def stats(self):
        j, u = ctypes.c_int64(), ctypes.c_int64()
        check(lib().wg_batcher_stats(self.h, ctypes.byref(j), ctypes.byref(u)))
        return j.value, u.value

    def close(self):
        if getattr(self, "h", None):
            lib().wg_batcher_destroy(self.h)
            self.h = None


class Job:
    """A decode job for U utterances (wg_job_*)."""

    def __init__(self, dec: WhisperDecoder, U: int, T: int, params: DecoderParams):
        self.dec, self.U, self.T, self.params = dec, U, T, params
        self.prompt = np.asarray(params.prompt, dtype=np.int32)
        self._cp = params.to_c()
        h = ctypes.c_void_p()
        check(lib().wg_job_create(dec.h, U, T, self.prompt.ctypes.data_as(c_int32_p), len(self.prompt),
                                  ctypes.byref(self._cp), ctypes.byref(h)), "job create")
        self.h = h
        self.max_tokens = max_tokens_for(params, dec.n_text_ctx)
        self._keep = None

    def upload(self, encoder_outs):
        arrs, ptrs = _enc_array(encoder_outs)
        self._keep = (arrs, ptrs)
        check(lib().wg_job_upload_encoder(self.h, ptrs), "upload")

    def utterance_device(self, u: int) -> int:
        dev = ctypes.c_int(-1)
        check(lib().wg_job_utterance_device(self.h, u, ctypes.byref(dev)))
        return dev.value

    def upload_device(self, ptrs: Sequence[int], stream: int = 0):
        """Encoder outputs already on the GPU: ptrs[u] is the device address of
        utterance u's [T, d] fp32 output on its device (utterance_device(u));
        the job's stream waits for `stream` (a cudaStream_t value, 0 = legacy
        default stream) before copying them device to device."""
        arr = (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])
        self._keep = arr
        check(lib().wg_job_upload_encoder_device(self.h, arr, ctypes.c_void_p(int(stream)) if stream else None),
              "upload")

    def start(self):
        check(lib().wg_job_start(self.h), "start")

    def step(self, n: int) -> bool:
        done = ctypes.c_int(0)
        check(lib().wg_job_step(self.h, n, ctypes.byref(done)), "step")
        return bool(done.value)

    def run(self):
        while not self.step(64):
            pass

    def result(self):
        stride = len(self.prompt) + self.max_tokens
        toks = np.zeros((self.U, stride), dtype=np.int32)
        lens = np.zeros(self.U, dtype=np.int32)
        scores = np.zeros(self.U, dtype=np.float32)
        check(lib().wg_job_result(self.h, toks.ctypes.data_as(c_int32_p), lens.ctypes.data_as(c_int32_p),
                                  scores.ctypes.data_as(c_float_p)), "result")
        return toks, lens, scores

    def beams(self):
        """Every hypothesis after the steps so far: tokens [U, B, P+max_tokens], lens and scores [U, B]."""
        B = max(1, int(self.params.beam_size))
        stride = len(self.prompt) + self.max_tokens
        toks = np.zeros((self.U, B, stride), dtype=np.int32)
        lens = np.zeros((self.U, B), dtype=np.int32)
        scores = np.zeros((self.U, B), dtype=np.float32)
        check(lib().wg_job_beams(self.h, toks.ctypes.data_as(c_int32_p), lens.ctypes.data_as(c_int32_p),
                                 scores.ctypes.data_as(c_float_p)), "beams")
        return toks, lens, scores

    def stats(self):
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().wg_job_stats(self.h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))
        return a.value, b.value, c.value

    def uses_step_kernel(self) -> bool:
        on = ctypes.c_int(0)
        check(lib().wg_job_uses_step_kernel(self.h, ctypes.byref(on)))
        return bool(on.value)

    def time_kernel(self, kclass: str, iters: int = 5):
        ms, nbytes = ctypes.c_double(), ctypes.c_double()
        check(lib().wg_job_time_kernel(self.h, KCLASS[kclass], iters, ctypes.byref(ms), ctypes.byref(nbytes)))
        return ms.value, nbytes.value

    def timer_start(self):
        check(lib().wg_job_timer(self.h, 0, None))

    def timer_stop(self) -> float:
        """Elapsed device milliseconds since timer_start (CUDA events on the job's streams)."""
        ms = ctypes.c_double()
        check(lib().wg_job_timer(self.h, 1, ctypes.byref(ms)))
        return ms.value

    def cancel(self):
        lib().wg_job_cancel(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().wg_job_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequant(qtype, raw: bytes, n: int) -> np.ndarray:
    qt = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    buf = np.frombuffer(bytes(raw), dtype=np.uint8).copy()
    out = np.empty(n, dtype=np.float32)
    check(lib().wg_dequant_test(qt, buf.ctypes.data, n, out.ctypes.data_as(c_float_p)), "dequant")
    return out


def matmul(qtype, raw: bytes, rows: int, cols: int, x: np.ndarray, path: int = 0) -> np.ndarray:
    qt = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    buf = np.frombuffer(bytes(raw), dtype=np.uint8).copy() if not isinstance(raw, np.ndarray) else raw
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((x.shape[0], rows), dtype=np.float32)
    check(lib().wg_matmul_test(qt, buf.ctypes.data, rows, cols, x.ctypes.data_as(c_float_p), x.shape[0],
                               out.ctypes.data_as(c_float_p), path), "matmul")
    return out


def sample(logits: np.ndarray, hist: np.ndarray, eot: int, params: DecoderParams, step: int = 0):
    """The token-selection kernels of one step on given logits [R, V] and
    histories [R, n] (wg_sample_test): greedy -> tokens [R]; beam -> (tokens
    [R, 5], log-probs [R, 5])."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    R, V = lg.shape
    h = np.ascontiguousarray(np.asarray(hist, dtype=np.int32).reshape(R, -1))
    cp = params.to_c()
    beam = params.beam_size > 1
    tok = np.zeros(R * 5 if beam else R, dtype=np.int32)
    lp = np.zeros(R * 5, dtype=np.float32)
    check(lib().wg_sample_test(lg.ctypes.data_as(c_float_p), R, V, h.ctypes.data_as(c_int32_p), h.shape[1],
                               int(eot), ctypes.byref(cp), int(step), tok.ctypes.data_as(c_int32_p),
                               lp.ctypes.data_as(c_float_p)), "sample")
    return (tok.reshape(R, 5), lp.reshape(R, 5)) if beam else tok


def quantize(qtype, data: np.ndarray) -> bytes:
    """Reference quantiser (internal/gguf/quant.go:99-232) over a flat run."""
    qt = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    data = np.ascontiguousarray(data, dtype=np.float32).ravel()
    nb = gen().wg_gen_row_bytes(qt, data.size)
    out = np.zeros(max(nb, 1), dtype=np.uint8)
    n = gen().wg_gen_quantize(qt, data.ctypes.data_as(c_float_p), data.size, out.ctypes.data)
    if n < 0:
        raise ValueError("unsupported qtype")
    return out[:n].tobytes()


def quantize_matrix(qtype, m: np.ndarray) -> bytes:
    qt = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
    m = np.ascontiguousarray(m, dtype=np.float32)
    rows, cols = m.shape
    rb = gen().wg_gen_row_bytes(qt, cols)
    out = np.zeros(rows * rb, dtype=np.uint8)
    if gen().wg_gen_quantize_matrix(qt, m.ctypes.data_as(c_float_p), rows, cols, out.ctypes.data) != 0:
        raise ValueError("unsupported qtype")
    return out.tobytes()
