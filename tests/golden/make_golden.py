"""Writes tests/golden/reference_kat.json: the known-answer vectors of the
reference's own tests for the decoder path, transcribed with their
file:line citations (paths inside the wxcdart/whisper.go module).

The reference is Go and cannot run here, so its test vectors are restated:
each entry rebuilds the test's input bytes exactly as the Go test does and
records the values the Go test asserts. When the REF environment variable
names a checkout of the reference, every citation is checked: the quoted
source fragment must appear on the cited line, so a transcription that drifts
from the reference fails loudly.
Run: REF=<whisper.go checkout> python tests/golden/make_golden.py
"""
import json
import os
import pathlib
import struct

HERE = pathlib.Path(__file__).resolve().parent
REF = pathlib.Path(os.environ["REF"]) if os.environ.get("REF") else None


def cite(path, line, fragment):
    """Checks that `fragment` occurs on line `line` of the reference file."""
    f = REF / path if REF else None
    if f is not None and f.exists():
        lines = f.read_text().splitlines()
        if fragment not in lines[line - 1]:
            raise SystemExit("citation mismatch: %s:%d does not contain %r" % (path, line, fragment))
    return "%s:%d" % (path, line)


def le16(v):
    return list(struct.pack("<H", v))


def le32(v):
    return list(struct.pack("<I", v))


kat = {"f16_to_f32": [], "dequant": [], "quant_roundtrip": [], "f16_conversion": [], "gelu": [],
       "layernorm": [], "attention": {}, "dot_q8": {}, "matmul_q8": {}, "matmul_all": {}, "decoder_tests": {}}

# ---- internal/gguf/gguf_test.go:155-186 TestF16ToF32 ---------------------------
G = "internal/gguf/gguf_test.go"
cite(G, 155, "func TestF16ToF32")
for h, want, line in [(0x0000, 0.0, 161), (0x8000, -0.0, 162), (0x3C00, 1.0, 163), (0x4000, 2.0, 164),
                      (0xBC00, -1.0, 165), (0x3800, 0.5, 166), (0x7C00, "inf", 167), (0xFC00, "-inf", 168),
                      (0x0001, 2.0 ** -24, 170), (0x03FF, 0x3FF * 2.0 ** -24, 172)]:
    cite(G, line, "0x%04X" % h)
    kat["f16_to_f32"].append({"h": h, "want": want, "src": "%s:%d" % (G, line)})
cite(G, 183, "0x7E00")
kat["f16_to_f32"].append({"h": 0x7E00, "want": "nan", "src": G + ":183"})

# ---- dequant known answers (gguf_test.go:190-309) ------------------------------
blk = [0] * 18
blk[0:2] = le16(0x3C00)
blk[2] = 0x9A
for i in range(3, 18):
    blk[i] = 0x88
cite(G, 196, "block[2] = 0x9A")
kat["dequant"].append({"qtype": "Q4_0", "block": blk, "n": 32,
                       "want": {"0": 2.0, "1": 1.0, **{str(i): 0.0 for i in range(2, 32)}},
                       "src": cite(G, 190, "func TestDequantQ4_0")})
blk = [0] * 20
blk[0:2] = le16(0x3C00)
blk[2:4] = le16(0x3800)
blk[4] = 0x23
cite(G, 221, "block[4] = 0x23")
kat["dequant"].append({"qtype": "Q4_1", "block": blk, "n": 32,
                       "want": {"0": 3.5, "1": 2.5, **{str(i): 0.5 for i in range(2, 32)}},
                       "src": cite(G, 216, "func TestDequantQ4_1")})
blk = [0] * 22
blk[0:2] = le16(0x3C00)
blk[2:6] = le32(0x00000003)
blk[6] = 0x04
for i in range(7, 22):
    blk[i] = 0x88
cite(G, 246, "block[6] = 0x04")
kat["dequant"].append({"qtype": "Q5_0", "block": blk, "n": 32, "want": {"0": 4.0, "1": 0.0, "2": -8.0},
                       "src": cite(G, 239, "func TestDequantQ5_0")})
blk = [0] * 24
blk[0:2] = le16(0x3C00)
blk[8] = 0x4F
cite(G, 275, "block[8] = 0x4F")
kat["dequant"].append({"qtype": "Q5_1", "block": blk, "n": 32, "want": {"0": 15.0, "1": 4.0},
                       "src": cite(G, 267, "func TestDequantQ5_1")})
blk = [0] * 34
blk[0:2] = le16(0x4000)
blk[2:6] = [1, 0xFF, 2, 0xFE]
cite(G, 292, "0xFF")
kat["dequant"].append({"qtype": "Q8_0", "block": blk, "n": 32,
                       "want": {"0": 2.0, "1": -2.0, "2": 4.0, "3": -4.0, **{str(i): 0.0 for i in range(4, 32)}},
                       "src": cite(G, 287, "func TestDequantQ8_0")})

# ---- internal/gguf/quant_test.go:11-85 TestQuantRoundTrip --------------------------
Q = "internal/gguf/quant_test.go"
cite(Q, 17, "input[i] = float32(i)/float32(blockSize-1)*2 - 1")
for qt, tol, line in [("Q4_0", 0.1, 30), ("Q4_1", 0.1, 36), ("Q5_0", 0.05, 42), ("Q5_1", 0.05, 48),
                      ("Q8_0", 0.01, 54), ("F16", 0.001, 60)]:
    cite(Q, line, "maxErr: %s" % tol)
    kat["quant_roundtrip"].append({"qtype": qt, "max_err": tol, "src": "%s:%d" % (Q, line)})
for name, val, tol, line in [("zero", 0.0, 0, 99), ("one", 1.0, 0, 100), ("neg_one", -1.0, 0, 101),
                             ("half", 0.5, 0, 102), ("max_f16", 65504.0, 0, 103),
                             ("min_f16_subnormal", 2.0 ** -24, 1e-30, 104)]:
    cite(Q, line, '"%s"' % name)
    kat["f16_conversion"].append({"name": name, "f32": val, "max_err": tol, "src": "%s:%d" % (Q, line)})

# ---- internal/ml/ops_test.go ---------------------------------------------------------
O = "internal/ml/ops_test.go"
for x, want, line in [(0, 0, 228), (1, 0.8413, 229), (-1, -0.1587, 230), (2, 1.9545, 231)]:
    cite(O, line, "{%s, %s}" % (x, want))
    kat["gelu"].append({"x": x, "want": want, "tol": 1e-3, "src": "%s:%d" % (O, line)})
cite(O, 279, "want := []float32{-1.68328, 0.10557, 1.89442, 3.68328}")
kat["layernorm"].append({"x": [1, 2, 3, 4], "w": [2, 2, 2, 2], "b": [1, 1, 1, 1],
                         "want": [-1.68328, 0.10557, 1.89442, 3.68328], "tol": 1e-3, "src": O + ":279"})
cite(O, 247, "x := From([]float32{1, 2, 3, 4}, 1, 4)")
kat["layernorm"].append({"x": [1, 2, 3, 4], "w": [1, 1, 1, 1], "b": [0, 0, 0, 0], "mean_tol": 1e-5,
                         "var_tol": 1e-4, "src": O + ":246-268"})
cite(O, 353, "qData := []float32{1, 0, 0, 0, 0, 1, 0, 0}")
kat["attention"] = {"q": [1, 0, 0, 0, 0, 1, 0, 0], "shape": [1, 2, 4], "causal_out0": [1, 0, 0, 0],
                    "causal_w10_w11_from": "softmax([0, 0.5])", "tol": 1e-4, "src": O + ":349-438"}

# ---- internal/ml/attention_test.go:9-60 -------------------------------------------
A = "internal/ml/attention_test.go"
cite(A, 57, "if maxAbs > 0.02")
kat["attention"]["fast_vs_exact"] = {"shape": [4, 32, 64], "max_abs": 0.02, "src": A + ":9-60"}

# ---- internal/ml/matmul_q8_test.go ----------------------------------------------------
M = "internal/ml/matmul_q8_test.go"
cite(M, 99, "f[i] = float32(i%7) - 3")
cite(M, 100, "g[i] = float32((i*3)%11) - 5")
kat["dot_q8"] = {"n": 64, "f": "i%7-3", "g": "(i*3)%11-5", "tol": 0.5, "src": M + ":95-114"}
cite(M, 121, "a.Data[i] = float32((i%13)-6) * 0.1")
cite(M, 125, "bF.Data[i] = float32((i%9)-4) * 0.2")
kat["matmul_q8"] = {"m": 2, "k": 64, "n": 3, "tol": 1.0, "src": M + ":116-149"}
cite(M, 156, "a.Data[i] = float32((i%17)-8) * 0.07")
cite(M, 160, "bF.Data[i] = float32((i%11)-5) * 0.11")
tols = {}
for qt, tol, line in [("Q4_0", 4.0, 169), ("Q4_1", 4.0, 170), ("Q5_0", 3.0, 171), ("Q5_1", 3.0, 172),
                      ("Q8_0", 1.0, 173)]:
    cite(M, line, "tol: %s" % tol)
    tols[qt] = tol
kat["matmul_all"] = {"m": 2, "k": 64, "n": 3, "tols": tols, "src": M + ":151-207"}

# ---- internal/model/decoder_test.go (smoke tests of the decoder) --------------------
D = "internal/model/decoder_test.go"
cite(D, 13, "testNVocab      = 51865")
cite(D, 101, "Prompt:      []int32{50258, 50259, 50357, 50363}")
kat["decoder_tests"] = {"n_vocab": 51865, "d": 4, "heads": 2, "layers": 1, "ctx": 128, "weight": 0.01,
                        "enc_len": 8, "enc_value": 0.01, "prompt": [50258, 50259, 50357, 50363],
                        "greedy_max_tokens": 5, "beam_size": 2, "temperature": 1.0, "src": D + ":12-180"}

out = HERE / "reference_kat.json"
out.write_text(json.dumps(kat, indent=1) + "\n")
print("wrote", out)
