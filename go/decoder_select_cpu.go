//go:build !cuda

package whisper

import (
	"github.com/whispergo/whisper.go/internal/gguf"
	"github.com/whispergo/whisper.go/internal/model"
	"github.com/whispergo/whisper.go/internal/vocab"
)

type vocabDecoder interface {
	model.Decoder
	SetVocabulary(v *vocab.Vocabulary)
}

// newDecoder is the reference's own decoder without -tags cuda.
func newDecoder(f gguf.FileLike, _ string) (vocabDecoder, error) { return model.NewDecoder(f) }
