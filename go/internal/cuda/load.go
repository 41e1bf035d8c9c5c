//go:build cuda

package cuda

/*
#include <stdlib.h>
#include <string.h>
#include "wg_decoder.h"
*/
import "C"

import (
	"context"
	"fmt"
	"strconv"
	"strings"
	"unsafe"

	"github.com/whispergo/whisper.go/internal/gguf"
)

func modelDims(m *C.wg_model) (nState, nCtx int) {
	var d, c C.int
	C.wg_model_info(m, nil, &d, nil, nil, &c)
	return int(d), int(c)
}

// hfDecoderName maps a whisper.cpp decoder tensor name to its Hugging Face
// name, the decoder half of internal/model/compat.go:31-148.
func hfDecoderName(name string) string {
	switch name {
	case "decoder.token_embedding.weight":
		return "model.decoder.embed_tokens.weight"
	case "decoder.positional_embedding":
		return "model.decoder.embed_positions.weight"
	case "decoder.ln.weight":
		return "model.decoder.layer_norm.weight"
	case "decoder.ln.bias":
		return "model.decoder.layer_norm.bias"
	}
	rest, ok := strings.CutPrefix(name, "decoder.blocks.")
	if !ok {
		return ""
	}
	idx, suffix, ok := strings.Cut(rest, ".")
	if _, err := strconv.Atoi(idx); !ok || err != nil {
		return ""
	}
	stem, leaf, ok := strings.Cut(suffix, ".weight")
	kind := "weight"
	if !ok || leaf != "" {
		if stem, ok = strings.CutSuffix(suffix, ".bias"); !ok {
			return ""
		}
		kind = "bias"
	}
	hf := map[string]string{
		"self_attn_ln": "self_attn_layer_norm", "self_attn.query": "self_attn.q_proj",
		"self_attn.key": "self_attn.k_proj", "self_attn.value": "self_attn.v_proj",
		"self_attn.out": "self_attn.out_proj", "cross_attn_ln": "encoder_attn_layer_norm",
		"cross_attn.query": "encoder_attn.q_proj", "cross_attn.key": "encoder_attn.k_proj",
		"cross_attn.value": "encoder_attn.v_proj", "cross_attn.out": "encoder_attn.out_proj",
		"mlp_ln": "final_layer_norm", "mlp.0": "fc1", "mlp.2": "fc2",
	}[stem]
	if hf == "" {
		return ""
	}
	return "model.decoder.layers." + idx + "." + hf + "." + kind
}

// descLoader builds a wg_model_desc in C memory from a gguf.FileLike.
type descLoader struct {
	f      gguf.FileLike
	desc   *C.wg_model_desc
	layers *C.wg_layer_desc
	allocs []unsafe.Pointer
}

func (l *descLoader) free() {
	for _, p := range l.allocs {
		C.free(p)
	}
	l.allocs = nil
}

func (l *descLoader) alloc(n int) unsafe.Pointer {
	p := C.malloc(C.size_t(n))
	l.allocs = append(l.allocs, p)
	return p
}

func (l *descLoader) resolve(name string) (string, bool) { // compat.go:15-29
	if _, ok := l.f.TensorType(name); ok {
		return name, true
	}
	if alt := hfDecoderName(name); alt != "" {
		if _, ok := l.f.TensorType(alt); ok {
			return alt, true
		}
	}
	return "", false
}

// vec returns an fp32 vector of n values in C memory (Tensor dequantises).
func (l *descLoader) vec(name string, n int) (*C.float, error) {
	r, ok := l.resolve(name)
	if !ok {
		return nil, fmt.Errorf("model: load tensor %q: not found", name)
	}
	data, _, err := l.f.Tensor(context.Background(), r)
	if err != nil || len(data) != n {
		return nil, fmt.Errorf("model: load tensor %q (resolved %q): want %d values", name, r, n)
	}
	p := l.alloc(4 * n)
	C.memcpy(p, unsafe.Pointer(&data[0]), C.size_t(4*n))
	return (*C.float)(p), nil
}

// mat fills m with a [rows, cols] matrix as TensorRaw returns it
// (quantised or dense); a dense matrix stored [cols, rows] is transposed
// (loadMatWeightAuto, compat.go:247-270).
func (l *descLoader) mat(name string, rows, cols int, m *C.wg_matrix) error {
	r, ok := l.resolve(name)
	if !ok {
		return fmt.Errorf("model: load tensor %q: not found", name)
	}
	raw, shape, qt, err := l.f.TensorRaw(context.Background(), r)
	if err != nil {
		return fmt.Errorf("model: load tensor %q (resolved %q): %w", name, r, err)
	}
	if len(shape) == 2 && shape[0] == rows && shape[1] == cols {
		p := l.alloc(len(raw))
		C.memcpy(p, unsafe.Pointer(&raw[0]), C.size_t(len(raw)))
		*m = C.wg_matrix{qtype: C.uint32_t(qt), rows: C.int32_t(rows), cols: C.int32_t(cols), data: p}
		return nil
	}
	if len(shape) == 2 && shape[0] == cols && shape[1] == rows {
		data, _, err := l.f.Tensor(context.Background(), r)
		if err != nil {
			return err
		}
		p := l.alloc(4 * rows * cols)
		dst := unsafe.Slice((*float32)(p), rows*cols)
		for i := 0; i < rows; i++ {
			for j := 0; j < cols; j++ {
				dst[i*cols+j] = data[j*rows+i]
			}
		}
		*m = C.wg_matrix{qtype: C.WG_QTYPE_F32, rows: C.int32_t(rows), cols: C.int32_t(cols), data: p}
		return nil
	}
	return fmt.Errorf("model: unsupported %s shape %v", name, shape)
}

func metaAny(f gguf.FileLike, keys ...string) int { // getMetaAny, compat.go:163-170
	for _, k := range keys {
		if v, ok := f.MetaUint32(k); ok {
			return int(v)
		}
	}
	return 0
}

func loadDesc(f gguf.FileLike) (*descLoader, error) {
	l := &descLoader{f: f}
	fail := func(err error) (*descLoader, error) { l.free(); return nil, err }
	nHead := metaAny(f, "whisper.decoder.attention.head_count")
	nLayer := metaAny(f, "whisper.decoder.layer_count")
	nCtx := metaAny(f, "whisper.decoder.context_length")
	nState := metaAny(f, "whisper.decoder.embedding_length")
	nVocab := metaAny(f, "whisper.vocab.size", "whisper.n_vocab")
	if nLayer == 0 { // decoder.go:108-112
		for {
			if _, ok := l.resolve(fmt.Sprintf("decoder.blocks.%d.self_attn.query.weight", nLayer)); !ok {
				break
			}
			nLayer++
		}
	}
	shape := func(name string) []int {
		r, ok := l.resolve(name)
		if !ok {
			return nil
		}
		_, s, _, err := f.TensorRaw(context.Background(), r)
		if err != nil {
			return nil
		}
		return s
	}
	if s := shape("decoder.blocks.0.self_attn.query.weight"); len(s) == 2 && s[0] == s[1] && s[0] > 0 {
		nState = s[0]
	}
	if nCtx == 0 || nState == 0 {
		s := shape("decoder.positional_embedding")
		if len(s) != 2 {
			return fail(fmt.Errorf("model: decoder: invalid positional embedding shape %v", s))
		}
		switch {
		case nState > 0 && s[0] == nState && s[1] != nState:
			nCtx = s[1]
		case nState > 0:
			nCtx = s[0]
		default:
			nCtx, nState = s[0], s[1]
		}
	}
	if nVocab == 0 {
		s := shape("decoder.token_embedding.weight")
		if len(s) != 2 {
			return fail(fmt.Errorf("model: decoder: invalid token embedding shape %v", s))
		}
		if s[1] == nState {
			nVocab = s[0]
		} else {
			nVocab = s[1]
		}
	}
	if nHead == 0 {
		if nState%64 != 0 {
			return fail(fmt.Errorf("model: decoder: cannot infer head count from embedding length %d", nState))
		}
		nHead = nState / 64
	}
	d := nState
	l.desc = (*C.wg_model_desc)(l.alloc(int(unsafe.Sizeof(C.wg_model_desc{}))))
	*l.desc = C.wg_model_desc{}
	l.layers = (*C.wg_layer_desc)(l.alloc(nLayer * int(unsafe.Sizeof(C.wg_layer_desc{}))))
	layers := unsafe.Slice(l.layers, nLayer)
	desc := l.desc
	desc.n_vocab, desc.n_state, desc.n_head = C.int32_t(nVocab), C.int32_t(d), C.int32_t(nHead)
	desc.n_layer, desc.n_text_ctx, desc.eot = C.int32_t(nLayer), C.int32_t(nCtx), 50256
	desc.layers = l.layers
	var err error
	if err = l.mat("decoder.token_embedding.weight", nVocab, d, &desc.token_embedding); err != nil {
		return fail(err)
	}
	if s := shape("decoder.positional_embedding"); len(s) == 2 && s[0] == d && s[1] == nCtx && d != nCtx {
		var m C.wg_matrix
		if err = l.mat("decoder.positional_embedding", nCtx, d, &m); err != nil {
			return fail(err)
		}
		desc.positional_embedding = (*C.float)(m.data)
	} else if desc.positional_embedding, err = l.vec("decoder.positional_embedding", nCtx*d); err != nil {
		return fail(err)
	}
	if desc.ln_w, err = l.vec("decoder.ln.weight", d); err != nil {
		return fail(err)
	}
	if desc.ln_b, err = l.vec("decoder.ln.bias", d); err != nil {
		return fail(err)
	}
	for i := range layers {
		b := &layers[i]
		p := fmt.Sprintf("decoder.blocks.%d.", i)
		vecs := []struct {
			name string
			n    int
			dst  **C.float
		}{
			{"self_attn_ln.weight", d, &b.self_ln_w}, {"self_attn_ln.bias", d, &b.self_ln_b},
			{"self_attn.query.bias", d, &b.self_q_b}, {"self_attn.value.bias", d, &b.self_v_b},
			{"self_attn.out.bias", d, &b.self_o_b}, {"cross_attn_ln.weight", d, &b.cross_ln_w},
			{"cross_attn_ln.bias", d, &b.cross_ln_b}, {"cross_attn.query.bias", d, &b.cross_q_b},
			{"cross_attn.value.bias", d, &b.cross_v_b}, {"cross_attn.out.bias", d, &b.cross_o_b},
			{"mlp_ln.weight", d, &b.mlp_ln_w}, {"mlp_ln.bias", d, &b.mlp_ln_b},
			{"mlp.0.bias", 4 * d, &b.mlp0_b}, {"mlp.2.bias", d, &b.mlp2_b},
		}
		for _, v := range vecs {
			if *v.dst, err = l.vec(p+v.name, v.n); err != nil {
				return fail(err)
			}
		}
		mats := []struct {
			name       string
			rows, cols int
			dst        *C.wg_matrix
		}{
			{"self_attn.query.weight", d, d, &b.self_q}, {"self_attn.key.weight", d, d, &b.self_k},
			{"self_attn.value.weight", d, d, &b.self_v}, {"self_attn.out.weight", d, d, &b.self_o},
			{"cross_attn.query.weight", d, d, &b.cross_q}, {"cross_attn.key.weight", d, d, &b.cross_k},
			{"cross_attn.value.weight", d, d, &b.cross_v}, {"cross_attn.out.weight", d, d, &b.cross_o},
			{"mlp.0.weight", 4 * d, d, &b.mlp0}, {"mlp.2.weight", d, 4 * d, &b.mlp2},
		}
		for _, m := range mats {
			if err = l.mat(p+m.name, m.rows, m.cols, m.dst); err != nil {
				return fail(err)
			}
		}
	}
	return l, nil
}
