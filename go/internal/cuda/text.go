//go:build cuda

package cuda

import (
	"bytes"
	"compress/gzip"

	"github.com/whispergo/whisper.go/internal/model"
	"github.com/whispergo/whisper.go/internal/vocab"
)

// compressionRatio is the byte length of s over its gzip length at the
// default level: the reference's retry test (decoder.go:1170-1183), with the
// same standard-library compressor.
func compressionRatio(s string) float32 {
	if s == "" {
		return 0
	}
	var buf bytes.Buffer
	w := gzip.NewWriter(&buf)
	_, _ = w.Write([]byte(s))
	_ = w.Close()
	if buf.Len() == 0 {
		return float32(len(s))
	}
	return float32(len(s)) / float32(buf.Len())
}

// collapseRuns replaces a unit of 1..maxUnit bytes that repeats minRepeats
// times in a row by one copy, scanning left to right on bytes
// (collapseRepeatedSubstrings, decoder.go:1188-1230).
func collapseRuns(s string, maxUnit, minRepeats int) string {
	if s == "" || maxUnit <= 0 || minRepeats <= 1 {
		return s
	}
	b := []byte(s)
	out := make([]byte, 0, len(b))
	for i := 0; i < len(b); {
		taken := false
		for l := 1; l <= maxUnit && l <= len(b)-i; l++ {
			unit := b[i : i+l]
			n := 1
			for j := i + l; j+l <= len(b) && n < minRepeats && bytes.Equal(b[j:j+l], unit); j += l {
				n++
			}
			if n >= minRepeats {
				out = append(out, unit...)
				i += l * n
				taken = true
				break
			}
		}
		if !taken {
			out = append(out, b[i])
			i++
		}
	}
	return string(out)
}

// tokensToSegments turns prompt + generated tokens into the one segment the
// reference returns (decoder.go:1415-1459): with a vocabulary, consecutive
// tokens with the same non-empty text are dropped and the text is the rest
// decoded, repeated substrings collapsed.
func tokensToSegments(tokens, prompt []int32, v *vocab.Vocabulary) []model.Segment {
	if len(tokens) < len(prompt) || len(tokens) == len(prompt) {
		return []model.Segment{}
	}
	seg := model.Segment{Tokens: make([]model.TokenData, 0, len(tokens)-len(prompt))}
	var last string
	kept := make([]vocab.Token, 0, len(tokens)-len(prompt))
	for _, t := range tokens[len(prompt):] {
		td := model.TokenData{ID: t}
		if v != nil {
			td.Text = v.DecodeToken(vocab.Token(t))
		}
		if td.Text != "" && td.Text == last {
			continue
		}
		last = td.Text
		seg.Tokens = append(seg.Tokens, td)
		kept = append(kept, vocab.Token(t))
	}
	if v != nil {
		seg.Text = collapseRuns(v.Decode(kept), 6, 3)
	}
	return []model.Segment{seg}
}
