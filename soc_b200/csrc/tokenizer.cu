// Host-side string pipeline: the bundle's byte-level BPE tokenizer and the Qwen3 chat
// template, so a prompt string becomes the token ids the device path consumes and
// generated ids become text again.  No GPU work.
//
// Behaviour restated from the reference (SongWooYoung/SoC, Mac/cpu):
//   TokenizerRuntimeLoader::LoadFromFile      src/runtime_assets.cpp:170-216
//   StartupValidator::ValidateTokenizerRuntime src/startup_validator.cpp:25-73
//   TokenizerRuntime::Encode / Decode          src/tokenizer_runtime.cpp (header tokenizer_runtime.h:17-18)
//   Qwen3TemplateBuilder::BuildPrompt          src/runtime_assets.cpp:221-258
// Encoding: added ("protected") tokens are matched longest-first where they occur; the text
// between them is split into pre-tokens (a whitespace run plus one run of ASCII letters,
// digits or other non-space bytes), each pre-token's bytes become byte-level symbols and
// the ranked merges are applied lowest rank first until none applies.
#include <algorithm>
#include <cctype>
#include <cstring>
#include <fstream>
#include <limits>
#include <sstream>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/soc_b200.h"
#include "common.cuh"
#include "json.hpp"

using socb::Error;
using socb::Json;
using socb::JsonReader;

struct soc_tokenizer {
    std::string im_start, im_end, think_start, think_end, default_system;
    std::unordered_map<std::string, int> id_of;
    std::unordered_map<int, std::string> token_of;
    std::unordered_set<int> added_ids;
    std::vector<std::string> added_longest_first;  // protected tokens, longest first
    std::vector<std::string> all_longest_first;    // every token (tokenizers without BPE)
    bool bpe = false;
    std::string unk, prefix, suffix;
    std::unordered_map<std::string, size_t> rank;  // "left\nright" -> merge order
    bool pre = false, pre_byte_level = false, pre_regex = true, pre_prefix_space = false;
    bool dec_byte_level = false, dec_bpe = false;
    std::string dec_suffix;
    std::vector<std::string> byte_sym;                     // byte -> symbol
    std::unordered_map<std::string, unsigned char> sym_byte;  // symbol -> byte
    long long vocab_size = 0;  // the file's vocab_size
    int max_id = -1;           // largest id over added tokens and vocab
};

namespace {

int tok_fail(int code, const std::string& m) {
    socb::set_last_error(m);
    return code;
}

template <typename F>
int tok_guard(F&& f) {
    try {
        f();
        return SOC_B200_OK;
    } catch (const Error& e) {
        return tok_fail(e.code, e.what());
    } catch (const std::exception& e) {
        return tok_fail(SOC_B200_ERR_FORMAT, e.what());
    }
}

[[noreturn]] void bad(const std::string& m) { throw Error(SOC_B200_ERR_FORMAT, m); }

std::string opt_string(const Json& v, const char* key) {
    return v.contains(key) && !v.at(key).is_null() ? v.at(key).as_string() : std::string();
}
bool opt_bool(const Json& v, const char* key, bool dflt) {
    return v.contains(key) && !v.at(key).is_null() ? v.at(key).as_bool() : dflt;
}

bool longer_then_smaller(const std::string& a, const std::string& b) {
    return a.size() != b.size() ? a.size() > b.size() : a < b;
}

void sort_unique(std::vector<std::string>& v) {
    std::sort(v.begin(), v.end(), longer_then_smaller);
    v.erase(std::unique(v.begin(), v.end()), v.end());
}

// Longest token of `list` (longest first) found at `at`, or "".
const std::string* longest_at(const std::vector<std::string>& list, const std::string& text, size_t at) {
    for (const std::string& t : list)
        if (!t.empty() && at + t.size() <= text.size() && text.compare(at, t.size(), t) == 0) return &t;
    return nullptr;
}

int id_or_throw(const soc_tokenizer& t, const std::string& token) {
    const auto it = t.id_of.find(token);
    if (it == t.id_of.end()) throw Error(SOC_B200_ERR_INVALID, "unknown token content: " + token);
    return it->second;
}

std::vector<std::string> pre_tokens(const soc_tokenizer& t, const std::string& s) {
    if (!t.pre || !t.pre_byte_level) return {s};
    std::vector<std::string> out;
    if (!t.pre_regex) {
        out.push_back(s);
    } else {
        auto sp = [&](size_t i) { return std::isspace(static_cast<unsigned char>(s[i])) != 0; };
        auto al = [&](size_t i) { return std::isalpha(static_cast<unsigned char>(s[i])) != 0; };
        auto dg = [&](size_t i) { return std::isdigit(static_cast<unsigned char>(s[i])) != 0; };
        size_t i = 0;
        while (i < s.size()) {
            const size_t start = i;
            while (i < s.size() && sp(i)) ++i;
            if (i == s.size()) {
                out.push_back(s.substr(start));
                break;
            }
            if (al(i)) {
                while (i < s.size() && al(i)) ++i;
            } else if (dg(i)) {
                while (i < s.size() && dg(i)) ++i;
            } else {
                while (i < s.size() && !sp(i) && !al(i) && !dg(i)) ++i;
            }
            out.push_back(s.substr(start, i - start));
        }
    }
    if (!out.empty() && t.pre_prefix_space && !out.front().empty() &&
        std::isspace(static_cast<unsigned char>(out.front().front())) == 0)
        out.front().insert(out.front().begin(), ' ');
    return out;
}

void encode_bpe_piece(const soc_tokenizer& t, const std::string& piece, std::vector<int>& ids) {
    const bool byte_level = t.pre_byte_level && !t.byte_sym.empty();
    std::vector<std::string> sym;
    sym.reserve(piece.size());
    for (size_t i = 0; i < piece.size(); ++i) {
        std::string s = byte_level ? t.byte_sym[static_cast<unsigned char>(piece[i])] : std::string(1, piece[i]);
        if (!t.prefix.empty() && i > 0) s = t.prefix + s;
        if (!t.suffix.empty() && i + 1 == piece.size()) s += t.suffix;
        sym.push_back(std::move(s));
    }
    while (sym.size() > 1 && !t.rank.empty()) {
        size_t best = sym.size(), best_rank = std::numeric_limits<size_t>::max();
        for (size_t i = 0; i + 1 < sym.size(); ++i) {
            const auto it = t.rank.find(sym[i] + '\n' + sym[i + 1]);
            if (it != t.rank.end() && it->second < best_rank) {
                best_rank = it->second;
                best = i;
            }
        }
        if (best == sym.size()) break;
        sym[best] += sym[best + 1];
        sym.erase(sym.begin() + static_cast<std::ptrdiff_t>(best) + 1);
    }
    for (const std::string& s : sym) {
        const auto it = t.id_of.find(s);
        if (it != t.id_of.end()) {
            ids.push_back(it->second);
        } else if (!t.unk.empty()) {
            ids.push_back(id_or_throw(t, t.unk));
        } else {
            throw Error(SOC_B200_ERR_INVALID, "tokenizer runtime cannot encode BPE symbol: " + s);
        }
    }
}

std::vector<int> encode(const soc_tokenizer& t, const std::string& text) {
    std::vector<int> ids;
    size_t at = 0;
    while (at < text.size()) {
        const std::string* m = longest_at(t.bpe ? t.added_longest_first : t.all_longest_first, text, at);
        if (m != nullptr) {
            ids.push_back(id_or_throw(t, *m));
            at += m->size();
            continue;
        }
        if (!t.bpe) throw Error(SOC_B200_ERR_INVALID, "tokenizer runtime cannot encode input at byte offset " + std::to_string(at));
        size_t next = text.size();
        for (const std::string& a : t.added_longest_first) {
            if (a.empty()) continue;
            const size_t p = text.find(a, at);
            if (p != std::string::npos && p < next) next = p;
        }
        for (const std::string& piece : pre_tokens(t, text.substr(at, next - at))) encode_bpe_piece(t, piece, ids);
        at = next;
    }
    return ids;
}

size_t utf8_width(unsigned char c) {
    if ((c & 0x80u) == 0) return 1;
    if ((c & 0xE0u) == 0xC0u) return 2;
    if ((c & 0xF0u) == 0xE0u) return 3;
    if ((c & 0xF8u) == 0xF0u) return 4;
    return 1;
}

std::string decode(const soc_tokenizer& t, const int32_t* ids, int n) {
    std::string text;
    bool first_model = true;
    for (int k = 0; k < n; ++k) {
        const auto it = t.token_of.find(ids[k]);
        if (it == t.token_of.end()) throw Error(SOC_B200_ERR_RANGE, "unknown token id: " + std::to_string(ids[k]));
        if (t.added_ids.count(ids[k])) {
            text += it->second;
            continue;
        }
        std::string tok = it->second;
        bool space = false;
        if (t.dec_bpe && !t.dec_suffix.empty() && tok.size() >= t.dec_suffix.size() &&
            tok.compare(tok.size() - t.dec_suffix.size(), t.dec_suffix.size(), t.dec_suffix) == 0) {
            tok.erase(tok.size() - t.dec_suffix.size());
            space = true;
        }
        if (!first_model && !t.prefix.empty() && tok.compare(0, t.prefix.size(), t.prefix) == 0)
            tok.erase(0, t.prefix.size());
        if (t.dec_byte_level && !t.sym_byte.empty()) {
            std::string bytes;
            for (size_t i = 0; i < tok.size();) {
                const size_t w = utf8_width(static_cast<unsigned char>(tok[i]));
                const std::string cp = tok.substr(i, w);
                const auto b = t.sym_byte.find(cp);
                if (b != t.sym_byte.end())
                    bytes.push_back(static_cast<char>(b->second));
                else
                    bytes += cp;
                i += w;
            }
            tok.swap(bytes);
        }
        if (space) tok.push_back(' ');
        text += tok;
        first_model = false;
    }
    return text;
}

std::string read_text(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error(SOC_B200_ERR_IO, "failed to open file: " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

void load(soc_tokenizer& t, const std::string& path) {
    Json root;
    try {
        root = JsonReader(read_text(path)).parse();
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        bad(e.what());
    }
    try {
        if (root.at("format").as_string() != "soc.cpp.tokenizer_runtime")
            bad("tokenizer runtime format must be soc.cpp.tokenizer_runtime");
        if (root.at("format_version").as_int64() != 1) bad("tokenizer runtime format_version must be 1");
        root.at("tokenizer_class").as_string();
        root.at("model_max_length").as_int64();
        t.vocab_size = root.at("vocab_size").as_int64();
        if (t.vocab_size <= 0) bad("tokenizer runtime vocab_size must be positive");
        const Json& tr = root.at("template_runtime");
        if (tr.at("type").as_string() != "qwen3") bad("tokenizer template runtime type must be qwen3");
        t.im_start = tr.at("im_start").as_string();
        t.im_end = tr.at("im_end").as_string();
        t.think_start = tr.at("think_start").as_string();
        t.think_end = tr.at("think_end").as_string();
        t.default_system = tr.at("default_system_prompt").as_string();
        for (const Json& a : root.at("added_tokens").as_array()) {
            const int id = static_cast<int>(a.at("id").as_int64());
            const std::string& c = a.at("content").as_string();
            t.id_of.emplace(c, id);
            t.token_of.emplace(id, c);
            t.added_ids.insert(id);
            t.max_id = std::max(t.max_id, id);
            t.added_longest_first.push_back(c);
            t.all_longest_first.push_back(c);
        }
        for (const Json& v : root.at("vocab").as_array()) {
            const int id = static_cast<int>(v.at("id").as_int64());
            const std::string& c = v.at("token").as_string();
            t.id_of.emplace(c, id);
            t.token_of.emplace(id, c);
            t.max_id = std::max(t.max_id, id);
            t.all_longest_first.push_back(c);
        }
        sort_unique(t.added_longest_first);
        sort_unique(t.all_longest_first);
        if (t.im_start.empty() || t.im_end.empty()) bad("tokenizer runtime must define chat boundary tokens");
        if (!t.id_of.count(t.im_start)) bad("tokenizer runtime is missing im_start token id");
        if (!t.id_of.count(t.im_end)) bad("tokenizer runtime is missing im_end token id");
        if (!t.id_of.count(t.think_start)) bad("tokenizer runtime is missing think_start token id");
        if (!t.id_of.count(t.think_end)) bad("tokenizer runtime is missing think_end token id");
        if (root.contains("bpe_model") && !root.at("bpe_model").is_null()) {
            const Json& b = root.at("bpe_model");
            t.bpe = true;
            if (b.at("type").as_string() != "bpe") bad("tokenizer bpe_model type must be bpe");
            t.unk = opt_string(b, "unk_token");
            t.prefix = opt_string(b, "continuing_subword_prefix");
            t.suffix = opt_string(b, "end_of_word_suffix");
            size_t r = 0;
            for (const Json& m : b.at("merges").as_array())
                t.rank.emplace(m.at("left").as_string() + '\n' + m.at("right").as_string(), r++);
            if (b.at("merges").as_array().empty()) bad("tokenizer bpe_model must define merges");
            if (!t.unk.empty() && !t.id_of.count(t.unk)) bad("tokenizer bpe_model unk_token must exist in tokenizer vocab");
        }
        if (root.contains("pre_tokenizer") && !root.at("pre_tokenizer").is_null()) {
            const Json& p = root.at("pre_tokenizer");
            t.pre = true;
            if (p.contains("byte_level") && !p.at("byte_level").is_null()) {
                const Json& bl = p.at("byte_level");
                t.pre_byte_level = opt_bool(bl, "enabled", true);
                t.pre_prefix_space = opt_bool(bl, "add_prefix_space", false);
                t.pre_regex = opt_bool(bl, "use_regex", true);
            }
            if (t.pre_byte_level && opt_string(p, "type").empty())
                bad("tokenizer pre_tokenizer must define a type when enabled");
        }
        if (root.contains("decoder") && !root.at("decoder").is_null()) {
            const Json& d = root.at("decoder");
            if (d.contains("byte_level") && !d.at("byte_level").is_null()) {
                const Json& bl = d.at("byte_level");
                t.dec_byte_level = opt_bool(bl, "enabled", true);
                if (bl.contains("byte_to_unicode") && !bl.at("byte_to_unicode").is_null())
                    for (const Json& m : bl.at("byte_to_unicode").as_array()) t.byte_sym.push_back(m.as_string());
                if (t.dec_byte_level && !t.byte_sym.empty() && t.byte_sym.size() != 256)
                    bad("tokenizer decoder byte_to_unicode mapping must contain 256 entries when provided");
                for (size_t b = 0; b < t.byte_sym.size(); ++b)
                    t.sym_byte.emplace(t.byte_sym[b], static_cast<unsigned char>(b));
            }
            if (d.contains("bpe") && !d.at("bpe").is_null()) {
                t.dec_bpe = opt_bool(d.at("bpe"), "enabled", true);
                t.dec_suffix = opt_string(d.at("bpe"), "suffix");
            }
        }
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        bad(e.what());
    }
}

int copy_out(const std::string& s, char* out, size_t cap, size_t* len) {
    if (len) *len = s.size();
    if (out && cap) std::memcpy(out, s.data(), std::min(cap, s.size()));
    if (s.size() > cap) return tok_fail(SOC_B200_ERR_CAPACITY, "output buffer too small");
    return SOC_B200_OK;
}

// ResolveRelativePath (Mac/cpu/src/runtime_assets.cpp): absolute paths stay, relative ones
// hang off the manifest's directory.
std::string manifest_relative(const std::string& manifest, const std::string& p) {
    if (!p.empty() && p[0] == '/') return p;
    const auto cut = manifest.find_last_of('/');
    return (cut == std::string::npos ? std::string() : manifest.substr(0, cut + 1)) + p;
}

// ReadOptionalInt / ReadOptionalSize / ReadOptionalFloat (Mac/cpu/src/runtime_pipeline.cpp:6-33):
// a missing key keeps the default; an integer given as an array takes its first element.
long long opt_int(const Json& o, const char* key, long long fallback, bool array_ok) {
    if (!o.is_object() || !o.contains(key)) return fallback;
    const Json& v = o.at(key);
    if (array_ok && v.is_array()) return v.as_array().empty() ? fallback : v.as_array().front().as_int64();
    return v.as_int64();
}

}  // namespace

extern "C" {

int soc_b200_manifest_generation_options(const char* manifest_path, soc_generation_options* out) {
    if (!manifest_path || !out) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    return tok_guard([&] {
        Json root;
        try {
            root = JsonReader(read_text(manifest_path)).parse();
        } catch (const Error&) {
            throw;
        } catch (const std::exception& e) {
            bad(e.what());
        }
        soc_generation_options o;
        o.max_new_tokens = 32;
        o.temperature = 1.0f;
        o.top_k = 1;
        o.eos_token_id = -1;
        o.max_sequence_length = 256;
        try {
            if (root.contains("generation_config")) {
                const Json& g = root.at("generation_config");
                o.max_new_tokens = static_cast<size_t>(opt_int(g, "max_new_tokens", 32, false));
                if (g.is_object() && g.contains("temperature"))
                    o.temperature = static_cast<float>(g.at("temperature").as_number());
                o.top_k = static_cast<size_t>(opt_int(g, "top_k", 1, false));
                o.eos_token_id = static_cast<int>(opt_int(g, "eos_token_id", -1, true));
                o.max_sequence_length = static_cast<size_t>(opt_int(g, "max_length", 256, false));
            }
        } catch (const Error&) {
            throw;
        } catch (const std::exception& e) {
            bad(e.what());
        }
        *out = o;
    });
}

int soc_b200_manifest_tokenizer_path(const char* manifest_path, char* out, size_t capacity, size_t* len) {
    if (!manifest_path) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    int rc = SOC_B200_OK;
    const int g = tok_guard([&] {
        Json root;
        try {
            root = JsonReader(read_text(manifest_path)).parse();
            if (!root.contains("tokenizer_runtime_file") || root.at("tokenizer_runtime_file").as_string().empty())
                bad("manifest must reference tokenizer_runtime_file");
        } catch (const Error&) {
            throw;
        } catch (const std::exception& e) {
            bad(e.what());
        }
        const std::string p = manifest_relative(manifest_path, root.at("tokenizer_runtime_file").as_string());
        rc = copy_out(p + std::string(1, '\0'), out, capacity, len);
        if (len) *len -= 1;
    });
    return g != SOC_B200_OK ? g : rc;
}

int soc_b200_tokenizer_check_model(const soc_tokenizer* t, long long model_vocab_size) {
    if (!t) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    if (t->vocab_size <= 0) return tok_fail(SOC_B200_ERR_FORMAT, "tokenizer vocab_size must be positive");
    if (t->vocab_size > model_vocab_size)
        return tok_fail(SOC_B200_ERR_FORMAT, "tokenizer vocab_size must not exceed qwen3 config vocab_size");
    if (t->max_id < 0 || t->max_id >= model_vocab_size)
        return tok_fail(SOC_B200_ERR_FORMAT, "tokenizer token ids must fit within qwen3 config vocab_size");
    return SOC_B200_OK;
}

int soc_b200_sampler_check(float temperature, size_t top_k) {
    if (!(temperature > 0.0f)) return tok_fail(SOC_B200_ERR_INVALID, "sampler temperature must be positive");
    if (top_k == 0) return tok_fail(SOC_B200_ERR_INVALID, "sampler top_k must be positive");
    return SOC_B200_OK;
}

int soc_b200_tokenizer_load(const char* path, soc_tokenizer** out) {
    if (!path || !out) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    auto t = new soc_tokenizer();
    const int rc = tok_guard([&] { load(*t, path); });
    if (rc != SOC_B200_OK) {
        delete t;
        return rc;
    }
    *out = t;
    return SOC_B200_OK;
}

void soc_b200_tokenizer_free(soc_tokenizer* t) { delete t; }

int soc_b200_tokenizer_encode(const soc_tokenizer* t, const char* text, size_t len, int32_t* ids, int capacity,
                              int* n_ids) {
    if (!t || (!text && len) || !n_ids) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    int rc = SOC_B200_OK;
    const int g = tok_guard([&] {
        const std::vector<int> v = encode(*t, std::string(text ? text : "", len));
        *n_ids = static_cast<int>(v.size());
        for (int i = 0; i < *n_ids && i < capacity && ids; ++i) ids[i] = v[i];
        if (*n_ids > capacity) rc = tok_fail(SOC_B200_ERR_CAPACITY, "token id buffer too small");
    });
    return g != SOC_B200_OK ? g : rc;
}

int soc_b200_tokenizer_decode(const soc_tokenizer* t, const int32_t* ids, int n, char* text, size_t capacity,
                              size_t* len) {
    if (!t || (!ids && n) || n < 0) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    int rc = SOC_B200_OK;
    const int g = tok_guard([&] { rc = copy_out(decode(*t, ids, n), text, capacity, len); });
    return g != SOC_B200_OK ? g : rc;
}

int soc_b200_chat_prompt(const soc_tokenizer* t, const char* const* roles, const char* const* contents, int n,
                         int add_generation_prompt, int enable_thinking, const char* system_prompt_override, char* out,
                         size_t capacity, size_t* len) {
    if (!t || n < 0 || (n && (!roles || !contents))) return tok_fail(SOC_B200_ERR_INVALID, "null argument");
    std::string turns;
    bool has_system = false;
    for (int i = 0; i < n; ++i) {
        if (!roles[i] || !contents[i]) return tok_fail(SOC_B200_ERR_INVALID, "null message");
        if (std::strcmp(roles[i], "system") == 0) has_system = true;
        turns += t->im_start + roles[i] + "\n" + contents[i] + t->im_end + "\n";
    }
    std::string prompt;
    if (!has_system) {
        const std::string sys =
            system_prompt_override && *system_prompt_override ? system_prompt_override : t->default_system;
        prompt = t->im_start + "system\n" + sys + t->im_end + "\n";
    }
    prompt += turns;
    if (add_generation_prompt) {
        prompt += t->im_start + "assistant\n";
        if (enable_thinking) prompt += t->think_start + "\n";
    }
    return copy_out(prompt, out, capacity, len);
}

}  // extern "C"
