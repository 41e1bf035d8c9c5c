//go:build cuda

// Package cuda runs whisper.go's decoder token loop on NVIDIA B200 GPUs
// through the C ABI of libwgdec.so (include/wg_decoder.h of the
// whisper.go_b200 repository). Decoder implements model.Decoder
// (internal/model/interfaces.go:22-25): the greedy and beam loops,
// forward, attention, the quantised matmuls and the samplers of
// internal/model/decoder.go all run on the device. There is no CPU path in
// this package; a missing device is an error.
//
// Build inside the whisper.go module (github.com/whispergo/whisper.go) with
//
//	CGO_CFLAGS="-I<repo>/include" \
//	CGO_LDFLAGS="-L<repo>/whisper.go_b200 -Wl,-rpath,<repo>/whisper.go_b200" \
//	go build -tags cuda ./...
package cuda

/*
#cgo LDFLAGS: -lwgdec
#include <stdlib.h>
#include "wg_decoder.h"
*/
import "C"

import (
	"context"
	"errors"
	"fmt"
	"unsafe"
)

// Status codes of the C ABI.
const (
	statusOK          = C.WG_OK
	statusInvalid     = C.WG_ERR_INVALID
	statusUnsupported = C.WG_ERR_UNSUPPORTED
	statusCancelled   = C.WG_ERR_CANCELLED
	statusTimeout     = C.WG_ERR_TIMEOUT
	statusNoDevice    = C.WG_ERR_NO_DEVICE
	statusDeviceFlag  = C.WG_ERR_DEVICE_FLAG
)

// ErrNoDevice is returned when no CUDA device can run the decoder.
var ErrNoDevice = errors.New("cuda: no CUDA device is available")

// Error is a failed call of the C ABI.
type Error struct {
	Status int
	Msg    string
}

func (e *Error) Error() string { return e.Msg }

// Is lets errors.Is(err, ErrNoDevice) hold for a missing device.
func (e *Error) Is(target error) bool { return target == ErrNoDevice && e.Status == statusNoDevice }

func lastError() string {
	var buf [1024]C.char
	C.wg_last_error(&buf[0], C.size_t(len(buf)))
	return C.GoString(&buf[0])
}

// check turns a status into an error with the reference's "model: decode:"
// prefix (decoder.go:442-457); cancellation wraps ctx's error so that
// errors.Is(err, context.Canceled) holds (decoder_test.go:145-151).
func check(ctx context.Context, rc C.int, what string) error {
	if rc == statusOK {
		return nil
	}
	msg := lastError()
	if rc == statusCancelled {
		cause := context.Canceled
		if ctx != nil && ctx.Err() != nil {
			cause = ctx.Err()
		}
		return fmt.Errorf("model: decode: cancelled: %w", cause)
	}
	if len(msg) < 6 || msg[:6] != "model:" {
		msg = "model: decode: " + what + ": " + msg
	}
	return &Error{Status: int(rc), Msg: msg}
}

// DeviceCount is the number of CUDA devices the library sees.
func DeviceCount() int {
	var n C.int
	C.wg_device_count(&n)
	return int(n)
}

func cParams(p decodeParams) C.wg_decode_params {
	var c C.wg_decode_params
	c.beam_size = C.int32_t(p.BeamSize)
	c.temperature = C.float(p.Temperature)
	c.attempt = C.int32_t(p.Attempt)
	c.logprob_thold = C.float(p.LogprobThold)
	c.no_speech_thold = C.float(p.NoSpeechThold)
	if p.NoFallback {
		c.no_fallback = 1
	}
	c.max_tokens = C.int32_t(p.MaxTokens)
	if p.SuppressNST {
		c.suppress_nst = 1
	}
	c.mode = C.WG_MODE_CORRECT
	if p.RefCompat {
		c.mode = C.WG_MODE_REF_COMPAT
	}
	c.seed = C.uint64_t(p.Seed)
	return c
}

func cInt32s(v []int32) *C.int32_t {
	if len(v) == 0 {
		return nil
	}
	return (*C.int32_t)(unsafe.Pointer(&v[0]))
}
