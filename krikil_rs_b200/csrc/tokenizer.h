// tokenizer.h -- byte-level BPE tokenizer read from a Hugging Face
// tokenizer.json, the text front end of the generation loop
// (src/tokenizer.rs:7-53 wraps the `tokenizers` crate 0.21.4 for this).
//
// Supported files: model "BPE" (merges as "a b" strings or [a, b] pairs, no
// dropout, no continuing-subword prefix / end-of-word suffix), pre-tokenizer
// "ByteLevel" with the GPT-2 split pattern, decoder "ByteLevel", no
// normalizer, added tokens matched literally (lstrip / rstrip honoured).
// Anything else is refused at load.  Host code only.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace krk {

class Tokenizer {
   public:
    // Reads and checks the file; nullptr and err set on failure.
    static std::unique_ptr<Tokenizer> from_file(const std::string& path, std::string& err);
    static std::unique_ptr<Tokenizer> from_json(const std::string& text, std::string& err);

    // Tokenizer::encode(text, add_special_tokens = false).ids(); false and
    // err set if text is not UTF-8.
    bool encode(const char* text, size_t len, std::vector<uint32_t>& ids, std::string& err) const;
    // Tokenizer::decode(ids, skip_special_tokens): unknown ids are dropped,
    // invalid UTF-8 becomes U+FFFD.
    std::string decode(const uint32_t* ids, size_t n, bool skip_special) const;
    // added tokens first, then the model vocabulary; -1 if absent
    int64_t token_to_id(const std::string& token) const;
    // distinct tokens of the vocabulary and the added tokens
    size_t vocab_size() const { return vocab_size_; }

   private:
    struct Added {
        std::string content;
        uint32_t id;
        bool special, lstrip, rstrip;
    };
    struct Merge {
        uint32_t rank, id;
    };
    void bpe_piece(const std::string& bytes, std::vector<uint32_t>& ids) const;
    void encode_segment(const std::vector<uint32_t>& cps, size_t lo, size_t hi, std::vector<uint32_t>& ids) const;

    std::unordered_map<std::string, uint32_t> vocab_;
    std::vector<std::string> id_to_token_;  // model vocabulary and added tokens ("" where none)
    std::vector<uint8_t> id_special_;       // 1 for special added tokens
    std::vector<uint8_t> id_known_;         // 1 where id_to_token_ holds a token
    std::unordered_map<uint64_t, Merge> merges_;  // (left id << 32 | right id) -> rank, merged id
    std::vector<Added> added_;
    int64_t byte_id_[256];  // vocabulary id of each byte's byte-level character (-1 if absent)
    bool add_prefix_space_ = false;
    size_t vocab_size_ = 0;
};

// Byte-level alphabet (GPT-2 bytes_to_unicode): the code point standing for byte b.
uint32_t byte_level_char(uint8_t b);
// UTF-8 of code point cp appended to s.
void append_utf8(std::string& s, uint32_t cp);
// String::from_utf8_lossy: each maximal invalid subsequence becomes U+FFFD.
std::string utf8_lossy(const std::string& bytes);

}  // namespace krk
