//go:build cuda

package whisper

// Decoder selection of whisper.New (whisper.go:153) when built with
// -tags cuda: the decoder token loop runs on the GPU (internal/cuda). There is
// no silent CPU fallback: without a usable device New fails, unless
// WHISPER_GO_CPU_DECODER=1 asks for the CPU decoder explicitly.

import (
	"fmt"
	"os"

	"github.com/whispergo/whisper.go/internal/cuda"
	"github.com/whispergo/whisper.go/internal/gguf"
	"github.com/whispergo/whisper.go/internal/model"
	"github.com/whispergo/whisper.go/internal/vocab"
)

type vocabDecoder interface {
	model.Decoder
	SetVocabulary(v *vocab.Vocabulary)
}

func newDecoder(f gguf.FileLike, modelPath string) (vocabDecoder, error) {
	if os.Getenv("WHISPER_GO_CPU_DECODER") == "1" {
		return model.NewDecoder(f)
	}
	if cuda.DeviceCount() == 0 {
		return nil, fmt.Errorf("load decoder: %w (set WHISPER_GO_CPU_DECODER=1 for the CPU decoder)", cuda.ErrNoDevice)
	}
	d, err := cuda.NewDecoderFromFile(modelPath, nil) // GGUF: mapped, uploaded without a host copy
	if err != nil {
		d, err = cuda.NewDecoder(f, nil) // legacy ggml files: through TensorRaw
	}
	if err != nil {
		return nil, err
	}
	// concurrent Transcribe calls and consecutive chunks share GPU jobs
	if err := d.EnableBatching(64, 2000); err != nil {
		d.Close()
		return nil, err
	}
	return d, nil
}
