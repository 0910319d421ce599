// TEST INFRASTRUCTURE ONLY (oracle): a stand-in definition of malkin::Tokenizer (the class declared in the
// reference's tokenizer.h), compiled into oracle/_ref/libmalkin_ref.so in place of tokenizer.cpp, whose byte-level
// BPE needs pcre2 (absent here). It exists so that malkin's Engine (engine.cpp) and ChatFormat (chat.cpp) compile
// unchanged and malkin's own continuous-batching / speculative decoding loop can check the device engine.
//
// Only what that loop reads from a tokenizer is given real behaviour, following tokenizer.h's contract: piece(id)
// is the GGUF token string (the synthetic models name token i "<ti>"), is_eog() marks the ids in
// tokenizer.ggml.eos_token_id / eot_token_id / eom_token_id, bos() / add_bos() come from the GGUF keys. encode()
// reads a text back as the concatenation of token strings ("<t12><t7>" -> 12, 7); there is no BPE.
#include <string>
#include <string_view>
#include <vector>

#include "tokenizer.h"

namespace malkin {

Tokenizer::Tokenizer(const GgufFile& f) {
  if (const auto* toks = f.get_str_array("tokenizer.ggml.tokens")) tokens_ = *toks;
  types_.assign(tokens_.size(), 1);
  eog_.assign(tokens_.size(), false);
  for (const char* key : {"tokenizer.ggml.eos_token_id", "tokenizer.ggml.eot_token_id", "tokenizer.ggml.eom_token_id"}) {
    const auto id = f.get_int(key);
    if (id && *id >= 0 && static_cast<size_t>(*id) < tokens_.size()) eog_[static_cast<size_t>(*id)] = true;
  }
  bos_ = static_cast<int32_t>(f.get_int("tokenizer.ggml.bos_token_id").value_or(-1));
  add_bos_ = f.get_int("tokenizer.ggml.add_bos_token").value_or(0) != 0 && bos_ >= 0;
  for (size_t i = 0; i < tokens_.size(); ++i) ids_.emplace(tokens_[i], static_cast<int32_t>(i));
}

Tokenizer::~Tokenizer() = default;

void Tokenizer::bpe(const std::string&, std::vector<int32_t>&) const {}

void Tokenizer::encode_plain(std::string_view text, std::vector<int32_t>& out) const {
  size_t at = 0;
  while (at < text.size()) {  // longest token string starting here
    size_t best = 0;
    int32_t id = -1;
    for (size_t len = 1; at + len <= text.size() && len <= 16; ++len) {
      const auto it = ids_.find(std::string(text.substr(at, len)));
      if (it != ids_.end()) best = len, id = it->second;
    }
    if (id < 0) break;
    out.push_back(id);
    at += best;
  }
}

std::vector<int32_t> Tokenizer::encode(std::string_view text, bool) const {
  std::vector<int32_t> out;
  encode_plain(text, out);
  return out;
}

std::string Tokenizer::piece(int32_t id) const {
  return id >= 0 && static_cast<size_t>(id) < tokens_.size() ? tokens_[static_cast<size_t>(id)] : std::string();
}

std::string Tokenizer::decode(const std::vector<int32_t>& ids) const {
  std::string s;
  for (int32_t id : ids) s += piece(id);
  return s;
}

bool Tokenizer::is_eog(int32_t id) const { return id >= 0 && static_cast<size_t>(id) < eog_.size() && eog_[static_cast<size_t>(id)]; }

bool Tokenizer::is_control(int32_t) const { return false; }

int32_t Tokenizer::find(const std::string& text) const {
  const auto it = ids_.find(text);
  return it == ids_.end() ? -1 : it->second;
}

}  // namespace malkin
