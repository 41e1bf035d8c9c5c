//go:build cuda

package cuda

import (
	"context"
	"errors"
	"os"
	"testing"

	"github.com/whispergo/whisper.go/internal/ml"
	"github.com/whispergo/whisper.go/internal/model"
)

// The reference decoder tests (internal/model/decoder_test.go:89-180) against
// the device decoder: a model file given by WG_TEST_GGUF (a whisper.go GGUF
// model), non-empty segments for greedy and beam search, and cancellation.
func testDecoder(t *testing.T) *Decoder {
	path := os.Getenv("WG_TEST_GGUF")
	if path == "" {
		t.Skip("WG_TEST_GGUF is not set")
	}
	if DeviceCount() == 0 {
		t.Skip("no CUDA device")
	}
	d, err := NewDecoderFromFile(path, nil)
	if err != nil {
		t.Fatal(err)
	}
	t.Cleanup(func() { d.Close() })
	return d
}

func encoderOut(d *Decoder, frames int) ml.Tensor {
	e := ml.New(frames, d.nState)
	for i := range e.Data {
		e.Data[i] = float32(i%7) * 0.01
	}
	return e
}

func TestDecodeGreedyAndBeam(t *testing.T) {
	d := testDecoder(t)
	for _, beam := range []int{1, 2, 5} {
		segs, err := d.Decode(context.Background(), encoderOut(d, 1500), model.DecoderParams{
			Prompt: []int32{50258, 50259, 50357, 50363}, BeamSize: beam, MaxTokens: 8,
		})
		if err != nil {
			t.Fatalf("beam %d: %v", beam, err)
		}
		if len(segs) != 1 || len(segs[0].Tokens) == 0 {
			t.Fatalf("beam %d: empty result %v", beam, segs)
		}
	}
}

func TestDecodeCancelled(t *testing.T) {
	d := testDecoder(t)
	ctx, cancel := context.WithCancel(context.Background())
	cancel()
	_, err := d.Decode(ctx, encoderOut(d, 1500), model.DecoderParams{Prompt: []int32{50258}, MaxTokens: 100})
	if !errors.Is(err, context.Canceled) {
		t.Fatalf("want context.Canceled, got %v", err)
	}
}

func TestEncoderShapeError(t *testing.T) {
	d := testDecoder(t)
	_, err := d.Decode(context.Background(), ml.New(10, d.nState+1), model.DecoderParams{Prompt: []int32{50258}})
	if err == nil {
		t.Fatal("want a shape error")
	}
}

func TestCollapseRuns(t *testing.T) {
	for in, want := range map[string]string{"tra tra tra tra": "tra tra", "aaaa": "aa", "abcabcabc!": "abc!", "hello": "hello"} {
		if got := collapseRuns(in, 6, 3); got != want {
			t.Errorf("collapseRuns(%q) = %q, want %q", in, got, want)
		}
	}
}
