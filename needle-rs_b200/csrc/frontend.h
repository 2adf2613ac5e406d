// frontend.h — the text front end of needle_run: SentencePiece BPE
// tokenizer, tool-JSON handling and the grammar-constrained decoding mask.
//
// Host code (C++17), no CUDA.  Each piece follows the reference's behaviour
// on the same inputs:
//   Vocab              crates/needle-infer/src/tokenizer.rs:31-246
//   to_snake_case      tokenizer.rs:248-292
//   tool JSON helpers  crates/needle-infer/src/constrained.rs:378-689,
//                      crates/needle-infer/src/engine.rs:354-546
//   Trie, JsonStateMachine, ConstrainedDecoder
//                      constrained.rs:15-375
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace ndl {
namespace text {

constexpr uint32_t kPadId = 0, kEosId = 1, kBosId = 2, kUnkId = 3, kToolCallId = 4, kToolsId = 5;

// True if s is well-formed UTF-8.
bool utf8_valid(const std::string &s);

// Vocabulary: one piece per line ("piece\tscore", or a bare piece in the
// legacy format), line index = token id.
class Vocab {
 public:
  void parse(const std::string &content);
  // Text -> token ids: trim, SentencePiece normalisation (leading U+2581,
  // whitespace runs -> one U+2581), then BPE merges by score (greedy
  // longest match when the file has no scores).
  std::vector<uint32_t> encode(const std::string &text) const;
  // Token ids -> text: pieces concatenated with U+2581 -> ' ', leading
  // whitespace removed.
  std::string decode_ids(const std::vector<uint32_t> &ids) const;
  size_t size() const { return id_to_piece_.size(); }
  const std::string &piece(uint32_t id) const { return id_to_piece_[id]; }
  // Piece text as the decoder emits it (U+2581 -> ' ').
  std::string piece_text(uint32_t id) const;
  bool has_scores() const { return !scores_.empty(); }

 private:
  std::vector<uint32_t> encode_bpe(const std::string &normalized) const;
  std::vector<uint32_t> encode_greedy(const std::string &bytes) const;
  bool lookup(const std::string &piece, uint32_t &id) const;

  std::vector<std::string> id_to_piece_;
  std::unordered_map<std::string, uint32_t> piece_to_id_;
  std::vector<float> scores_;  // empty: legacy vocabulary, greedy encoding
  size_t max_piece_bytes_ = 0;
};

std::string to_snake_case(const std::string &name);

struct ToolDef {
  std::string name, snake_name;
  std::vector<std::string> param_keys;
};
std::vector<ToolDef> parse_tools_json(const std::string &json);
// Tool names -> snake_case inside the tools JSON (the form the model saw in
// training), whitespace outside strings removed, and the reverse rename on
// the model's output.
std::string normalize_tools_json(const std::string &json, const std::vector<ToolDef> &defs);
std::string compact_json(const std::string &s);
std::string restore_tool_names(const std::string &text, const std::vector<ToolDef> &defs);

class Trie {
 public:
  Trie();
  void insert(const std::string &s);
  // Node reached from `node` by the bytes of s, or -1.
  int advance(int node, const std::string &s) const;
  // A token's bytes are a valid continuation from `node`: every byte before
  // the first '"' follows a child edge, and a '"' may only come at a terminal
  // node.
  bool token_valid(const std::string &bytes, int node) const;

 private:
  struct Node {
    std::unordered_map<uint8_t, int> children;
    bool terminal = false;
  };
  std::vector<Node> nodes_;
};

enum class JsonState { Free, InName, InArgKey };

// Position in the model's compact JSON output: the tool name after
// "name":" (outside the arguments object) and each argument key after {" or
// ," at the arguments object's depth are constrained regions.
class JsonStateMachine {
 public:
  void feed_byte(uint8_t b);
  void feed(const std::string &bytes) {
    for (unsigned char b : bytes) feed_byte(b);
  }
  JsonState state = JsonState::Free;
  std::string current_function;  // tool name captured when leaving InName
  std::string constrained_buf;   // bytes of the current constrained region

 private:
  void push_tail(uint8_t b);
  bool tail_ends_with(const char *pat, size_t n) const;
  bool in_arguments_ = false, in_string_ = false, prev_escape_ = false;
  size_t arguments_depth_ = 0, nesting_depth_ = 0;
  std::string tail_;  // the last 13 output bytes
};

class ConstrainedDecoder {
 public:
  ConstrainedDecoder(const std::vector<ToolDef> &tools, const Vocab &vocab);
  // Advance past an emitted token.
  void update(uint32_t token);
  void feed_bytes(const std::string &bytes) { sm_.feed(bytes); }
  // Allowed-token bitmap for the next step: bit v of word v/64 set = token v
  // allowed (additive 0), clear = additive -1e9.  Returns false when the
  // step is unconstrained (every token allowed: Free state, off-trie prefix,
  // unknown tool, or no token valid).
  bool mask(size_t vocab_size, std::vector<uint64_t> &bits);
  const JsonStateMachine &state_machine() const { return sm_; }

 private:
  bool trie_mask(const Trie &trie, int trie_id, int node, size_t vocab_size, std::vector<uint64_t> &bits);

  Trie name_trie_;
  std::vector<Trie> param_tries_;
  std::unordered_map<std::string, int> param_index_;  // snake name -> param_tries_ index
  std::vector<std::string> token_texts_;
  JsonStateMachine sm_;
  // bitmaps already built, by (trie, node)
  std::unordered_map<uint64_t, std::pair<bool, std::vector<uint64_t>>> cache_;
  size_t cache_vocab_ = 0;  // vocab_size the cached bitmaps were built for
};

}  // namespace text
}  // namespace ndl
