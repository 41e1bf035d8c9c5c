//go:build cuda

package cuda

/*
#include <stdlib.h>
#include "wg_decoder.h"
*/
import "C"

import (
	"context"
	"fmt"
	"runtime"
	"sync"
	"unsafe"

	"github.com/whispergo/whisper.go/internal/gguf"
	"github.com/whispergo/whisper.go/internal/ml"
	"github.com/whispergo/whisper.go/internal/model"
	"github.com/whispergo/whisper.go/internal/vocab"
)

// decodeParams is model.DecoderParams plus the switches of the device decoder.
type decodeParams struct {
	model.DecoderParams
	Attempt   int
	RefCompat bool   // the reference's literal semantics (decoder.go:750-757, attention.go:250-256)
	Seed      uint64 // top-p draws (the reference's are unseeded)
}

// Decoder is the device decoder. It is safe for concurrent use: every
// Decode runs its own job (or, with EnableBatching, shares a job with
// concurrent calls).
type Decoder struct {
	m      *C.wg_model
	nState int
	nCtx   int

	mu      sync.RWMutex
	vocab   *vocab.Vocabulary
	batcher *C.wg_batcher

	// RefCompat selects the reference's literal decoding semantics
	// (WG_MODE_REF_COMPAT); the default is standard Whisper decoding.
	RefCompat bool
	// Seed of the top-p fallback draws.
	Seed uint64
}

var _ model.Decoder = (*Decoder)(nil)

// NewDecoderFromFile loads the decoder of a GGUF model file onto the listed
// devices (nil: device 0): the file is mapped and its quantised blocks are
// uploaded without a host copy (wg_model_create_from_gguf).
func NewDecoderFromFile(path string, devices []int) (*Decoder, error) {
	cpath := C.CString(path)
	defer C.free(unsafe.Pointer(cpath))
	devs, n := cDevices(devices)
	if devs != nil {
		defer C.free(unsafe.Pointer(devs))
	}
	var m *C.wg_model
	if err := check(nil, C.wg_model_create_from_gguf(cpath, devs, n, &m), "load"); err != nil {
		return nil, fmt.Errorf("model: decoder: %w", err)
	}
	return newDecoder(m), nil
}

// NewDecoder loads the decoder from any gguf.FileLike (a legacy ggml file
// included): the tensors are read with TensorRaw under the names NewDecoder
// uses (internal/model/decoder.go:97-303, compat.go:15-29), copied to C
// memory for the upload, and freed once they are on the devices.
func NewDecoder(f gguf.FileLike, devices []int) (*Decoder, error) {
	ld, err := loadDesc(f)
	if err != nil {
		return nil, err
	}
	defer ld.free()
	devs, n := cDevices(devices)
	if devs != nil {
		defer C.free(unsafe.Pointer(devs))
	}
	var m *C.wg_model
	if err := check(nil, C.wg_model_create(ld.desc, devs, n, &m), "load"); err != nil {
		return nil, fmt.Errorf("model: decoder: %w", err)
	}
	return newDecoder(m), nil
}

func newDecoder(m *C.wg_model) *Decoder {
	d := &Decoder{m: m}
	// hyper-parameters for argument checks
	d.nState, d.nCtx = modelDims(m)
	runtime.SetFinalizer(d, (*Decoder).Close)
	return d
}

// SetVocabulary attaches the vocabulary (decoder.go:85-95): token texts in
// the segments, the compression-ratio retry, and the vocabulary's EOT id.
func (d *Decoder) SetVocabulary(v *vocab.Vocabulary) {
	d.mu.Lock()
	defer d.mu.Unlock()
	d.vocab = v
	if v != nil && v.Special().EOT >= 0 {
		C.wg_model_set_eot(d.m, C.int(v.Special().EOT))
	}
}

// EnableBatching gathers concurrent single-utterance Decode calls with equal
// prompts and parameters into shared jobs of up to maxUtterances, waiting at
// most window for company (wg_batcher_*; pipeline.go:90-193 decodes chunk by
// chunk, and Context.Transcribe may run concurrently, whisper.go:24).
func (d *Decoder) EnableBatching(maxUtterances int, windowMicros int) error {
	d.mu.Lock()
	defer d.mu.Unlock()
	if d.batcher != nil {
		return nil
	}
	return check(nil, C.wg_batcher_create(d.m, C.int(maxUtterances), C.int(windowMicros), &d.batcher), "batcher")
}

// Close releases the device memory.
func (d *Decoder) Close() error {
	d.mu.Lock()
	defer d.mu.Unlock()
	if d.batcher != nil {
		C.wg_batcher_destroy(d.batcher)
		d.batcher = nil
	}
	if d.m != nil {
		C.wg_model_destroy(d.m)
		d.m = nil
	}
	return nil
}

// Decode implements model.Decoder (interfaces.go:22-25).
func (d *Decoder) Decode(ctx context.Context, encoderOut ml.Tensor, params model.DecoderParams) ([]model.Segment, error) {
	out, err := d.DecodeBatch(ctx, []ml.Tensor{encoderOut}, params)
	if err != nil {
		return nil, err
	}
	return out[0], nil
}

// DecodeBatch decodes several utterances with the same parameters in one
// job (more rows per token step for the same weight stream). With a
// vocabulary, an utterance whose text compresses by more than 2.4 is decoded
// again at temperature + 0.2 * attempt, up to 3 attempts, unless NoFallback
// (decoder.go:433-515, :536-716); the retries of a batch share a job too.
func (d *Decoder) DecodeBatch(ctx context.Context, encs []ml.Tensor, params model.DecoderParams) ([][]model.Segment, error) {
	for _, e := range encs {
		if len(e.Shape) != 2 || e.Shape[1] != d.nState {
			return nil, fmt.Errorf("model: decoder: encoder output must be [T, %d], got %v", d.nState, e.Shape)
		}
	}
	if len(encs) == 0 {
		return nil, nil
	}
	d.mu.RLock()
	v := d.vocab
	d.mu.RUnlock()
	attempts := 1
	if v != nil {
		attempts = 3
	}
	final := make([][]int32, len(encs))
	pending := make([]int, len(encs))
	for i := range pending {
		pending[i] = i
	}
	for attempt := 0; attempt < attempts && len(pending) > 0; attempt++ {
		sub := make([]ml.Tensor, len(pending))
		for k, u := range pending {
			sub[k] = encs[u]
		}
		p := decodeParams{DecoderParams: params, Attempt: attempt, RefCompat: d.RefCompat, Seed: d.Seed}
		toks, err := d.run(ctx, sub, p)
		if err != nil {
			return nil, err
		}
		var retry []int
		for k, u := range pending {
			final[u] = toks[k]
			if v == nil || len(toks[k]) <= len(params.Prompt) {
				continue
			}
			gen := toks[k][len(params.Prompt):]
			vt := make([]vocab.Token, len(gen))
			for i, t := range gen {
				vt[i] = vocab.Token(t)
			}
			text := v.Decode(vt)
			if text != "" && compressionRatio(text) > 2.4 && attempt < attempts-1 && !params.NoFallback {
				retry = append(retry, u)
			}
		}
		pending = retry
	}
	out := make([][]model.Segment, len(encs))
	for u := range encs {
		out[u] = tokensToSegments(final[u], params.Prompt, v)
	}
	return out, nil
}

// run decodes the utterances of encs in one job (or through the batcher for
// a single utterance) and returns prompt + generated tokens of each.
func (d *Decoder) run(ctx context.Context, encs []ml.Tensor, p decodeParams) ([][]int32, error) {
	if len(p.Prompt) == 0 {
		return nil, fmt.Errorf("model: decode: forward: no tokens in state")
	}
	if err := ctx.Err(); err != nil {
		return nil, fmt.Errorf("model: decode: cancelled: %w", err)
	}
	cp := cParams(p)
	T := encs[0].Shape[0]
	maxTok := p.MaxTokens // decoder.go:421-430
	if maxTok <= 0 {
		maxTok = d.nCtx
	}
	if c := d.nCtx - len(p.Prompt); c < maxTok {
		maxTok = c
	}
	if maxTok < 0 {
		maxTok = 0
	}
	stride := len(p.Prompt) + maxTok
	d.mu.RLock()
	b := d.batcher
	d.mu.RUnlock()
	if b != nil && len(encs) == 1 && encs[0].Shape[0] == T {
		return d.runBatched(ctx, b, encs[0], p, &cp, stride)
	}
	var job *C.wg_job
	if err := check(ctx, C.wg_job_create(d.m, C.int(len(encs)), C.int(T), cInt32s(p.Prompt), C.int(len(p.Prompt)), &cp, &job), "job"); err != nil {
		return nil, err
	}
	defer C.wg_job_destroy(job)
	for u, e := range encs {
		if e.Shape[0] != T {
			return nil, fmt.Errorf("model: decoder: every encoder output of a batch must have %d frames, got %v", T, e.Shape)
		}
		if err := check(ctx, C.wg_job_upload_encoder_one(job, C.int(u), (*C.float)(unsafe.Pointer(&e.Data[0]))), "upload"); err != nil {
			return nil, err
		}
	}
	if err := check(ctx, C.wg_job_start(job), "start"); err != nil {
		return nil, err
	}
	for done := C.int(0); done == 0; {
		if ctx.Err() != nil { // checked between token-step batches, like the reference's loop (decoder.go:442)
			C.wg_job_cancel(job)
		}
		if err := check(ctx, C.wg_job_step(job, 16, &done), "step"); err != nil {
			return nil, err
		}
	}
	toks := make([]int32, len(encs)*stride)
	lens := make([]int32, len(encs))
	scores := make([]float32, len(encs))
	if err := check(ctx, C.wg_job_result(job, cInt32s(toks), cInt32s(lens), (*C.float)(unsafe.Pointer(&scores[0]))), "result"); err != nil {
		return nil, err
	}
	out := make([][]int32, len(encs))
	for u := range out {
		out[u] = append([]int32(nil), toks[u*stride:u*stride+int(lens[u])]...)
	}
	return out, nil
}

func (d *Decoder) runBatched(ctx context.Context, b *C.wg_batcher, e ml.Tensor, p decodeParams, cp *C.wg_decode_params, stride int) ([][]int32, error) {
	cancel := (*C.int)(C.malloc(C.size_t(unsafe.Sizeof(C.int(0)))))
	*cancel = 0
	defer C.free(unsafe.Pointer(cancel))
	stop := make(chan struct{})
	defer close(stop)
	go func() { // ctx.Done() -> the request's cancel flag, polled between token steps
		select {
		case <-ctx.Done():
			*(*C.int)(unsafe.Pointer(cancel)) = 1
		case <-stop:
		}
	}()
	toks := make([]int32, stride)
	var n C.int32_t
	var score C.float
	rc := C.wg_batcher_decode(b, (*C.float)(unsafe.Pointer(&e.Data[0])), C.int(e.Shape[0]), cInt32s(p.Prompt),
		C.int(len(p.Prompt)), cp, (*C.int)(unsafe.Pointer(cancel)), cInt32s(toks), C.int(stride), &n, &score)
	if err := check(ctx, rc, "decode"); err != nil {
		return nil, err
	}
	return [][]int32{toks[:int(n)]}, nil
}

func cDevices(devices []int) (*C.int, C.int) {
	if len(devices) == 0 {
		return nil, 0
	}
	p := (*C.int)(C.malloc(C.size_t(len(devices)) * C.size_t(unsafe.Sizeof(C.int(0)))))
	s := unsafe.Slice(p, len(devices))
	for i, v := range devices {
		s[i] = C.int(v)
	}
	return p, C.int(len(devices))
}
