// ref_detok_shim.cpp -- TEST INFRASTRUCTURE ONLY: a C entry point around the
// reference's own detokenize (src/sentencepiece_bpe.cpp:9-37), compiled from
// the reference's sources into oracle/_ref/ (see Makefile target `ref`). Tests
// use it to pin orc_detokenize and pk_detokenize against the reference itself.

#include "sentencepiece_bpe.h"

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

extern "C" int64_t ref_detokenize(const uint8_t * bytes, const int64_t * offsets, int32_t n_pieces, int32_t blank_id,
                                  int32_t bos_id, int32_t eos_id, int32_t pad_id, const int32_t * tokens,
                                  int64_t n_tokens, char * text, int64_t cap) {
    parakeet::BpeVocab v;
    v.pieces.reserve((size_t) n_pieces);
    for (int32_t i = 0; i < n_pieces; ++i)
        v.pieces.emplace_back(reinterpret_cast<const char *>(bytes) + offsets[i], (size_t) (offsets[i + 1] - offsets[i]));
    v.blank_id = blank_id;
    v.bos_id = bos_id;
    v.eos_id = eos_id;
    v.pad_id = pad_id;
    const std::vector<int32_t> ids(tokens, tokens + n_tokens);
    const std::string out = parakeet::detokenize(v, ids);
    if (text) std::memcpy(text, out.data(), (size_t) (cap < (int64_t) out.size() ? cap : (int64_t) out.size()));
    return (int64_t) out.size();
}
