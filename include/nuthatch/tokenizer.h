// GPT-2 byte-level BPE tokenizer of OLMoE GGUF files (model "gpt2", pre
// "olmo"): the drop-in for the reference's src/tokenizer/tokenizer.h:13-44,
// same names and behaviour, without PCRE2 (this build splits the text with
// its own matcher of the same pattern over Unicode category tables).
//
// Encode: the text is cut into chunks by the OLMo pre-split pattern
//   's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)
// searched left to right, each match starting the next search at its end
// (tokenizer.cc:165-186).  Text no alternative matches is skipped, as the
// reference's search skips it (a lone non-space whitespace character before
// a non-space, e.g. the "\n" of "a\nb", yields no id).  \s is U+0009..U+000D
// and the Unicode separators (Zs, Zl, Zp).  Each chunk's bytes map to GPT-2's
// byte-level characters and the merges apply lowest rank first, leftmost
// among equal ranks (tokenizer.cc:129-157); a final symbol missing from the
// vocabulary yields no id.  Text that is not valid UTF-8 yields no ids.
// Decode: ids outside the vocabulary are skipped; each vocabulary string's
// characters map back to bytes (tokenizer.cc:188-200).
#ifndef NUTHATCH_B200_TOKENIZER_H_
#define NUTHATCH_B200_TOKENIZER_H_

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace nuthatch {

class Tokenizer {
 public:
  // Vocabulary from the GGUF key tokenizer.ggml.tokens (a string array,
  // required) and merges from tokenizer.ggml.merges (optional: without them
  // the tokenizer only decodes well).  nullptr on a missing or unreadable
  // file or a missing vocabulary (tokenizer.cc:69-90).
  static std::unique_ptr<Tokenizer> Load(const std::string& path);
  // The same from in-memory lists (tests and callers with their own files).
  static std::unique_ptr<Tokenizer> FromLists(std::vector<std::string> vocab, std::vector<std::string> merges);
  ~Tokenizer();

  Tokenizer(const Tokenizer&) = delete;
  Tokenizer& operator=(const Tokenizer&) = delete;

  std::vector<int32_t> Encode(const std::string& text) const;
  std::string Decode(const std::vector<int32_t>& ids) const;

  int64_t vocab_size() const { return static_cast<int64_t>(vocab_.size()); }
  // The vocabulary string of id (byte-level form); empty for ids outside it.
  const std::string& token(int32_t id) const;

  // The pre-split chunks of text as [begin, end) byte offsets (the first
  // stage of Encode; empty for text that is not valid UTF-8).
  static std::vector<std::pair<size_t, size_t>> Split(const std::string& text);

 private:
  Tokenizer(std::vector<std::string> vocab, std::vector<std::string> merges);
  void EncodeChunk(const char* p, size_t n, std::vector<int32_t>* out) const;

  // Symbols (every string the merges can form, and the vocabulary) are
  // interned as integers: a merge "A B" of rank r is the pair (A, B) ->
  // (r, AB).  Byte-level symbols never hold U+0020, so a merge string with
  // other than one space can never apply and is left out.
  std::vector<std::string> vocab_;
  std::vector<int32_t> sym_id_;                               // symbol -> vocabulary id or -1
  std::unordered_map<uint64_t, std::pair<int, int>> merge_;  // (A << 32 | B) -> (rank, AB)
  int byte_sym_[256];                                         // byte -> symbol of its byte-level character
  std::unordered_map<uint32_t, uint8_t> char_byte_;           // byte-level code point -> byte
  // Ids of recently seen chunks (words repeat); bounded, guarded for
  // concurrent Encode calls.
  mutable std::mutex cache_mu_;
  mutable std::unordered_map<std::string, std::vector<int32_t>> cache_;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_TOKENIZER_H_
