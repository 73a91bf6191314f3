// capi.cu -- the reference's public C ABI (include/npu_engine.h) over the B200 engine, plus
// the embedding pipeline's front end.
//
// Replaces rust/npu-capi/src/lib.rs:22-214 and, behind it, npu_engine::Model
// (rust/npu-engine/src/api.rs:44-100), the scenario manifest (rust/npu-engine/src/config.rs),
// the embed pipeline (bert/mod.rs:24-46: WordPiece frontend bert/frontend.rs:29-35, encoder,
// head bert/head.rs:20-47) and the npy weight store (bert/weights.rs:25-70).
//
// * Scenario TOML: the subset the reference's manifests use (tables, `key = value` with
//   strings, integers, floats, booleans, `#` comments).  Required fields as in config.rs:
//   scenario.kind / name; model.hidden / ff / n_heads / head_dim / n_layers / max_seq.
// * Weights: the legacy npy directory (artifacts.weights): emb/{word_emb, pos_emb, type_emb,
//   emb_ln_w, emb_ln_b}.npy and L{i}/{q_w, q_b, k_w, k_b, v_w, v_b, attn_out_w, attn_out_b,
//   attn_ln_w, attn_ln_b, ffn1_w, ffn1_b, ffn2_w, ffn2_b, out_ln_w, out_ln_b}.npy, linear
//   weights [in, out] f32 little-endian C order.
// * Tokenizer (artifacts.tokenizer): a HuggingFace tokenizer.json with a WordPiece model, or a
//   vocab.txt.  The BERT uncased pipeline is restated here: clean text, split CJK characters,
//   whitespace split, lower case + accent stripping, punctuation split, then greedy
//   longest-match-first WordPiece with "##" continuations (max 100 characters per word, else
//   [UNK]); [CLS] ... [SEP]; truncated to model.max_seq.  Lower-casing and accent stripping
//   cover ASCII and Latin-1; other code points pass through unchanged.
// * The encoder and head run on the GPU (xdna_bert_*).  ASR scenarios whose name contains
//   "whisper" run the Whisper pipeline of asr.cu behind npu_transcribe.
// * The control plane (npu_runtime_*) lives in runtime.cu and loads models through
//   npu_model_load_on, one replica per GPU.
#include <cuda_runtime.h>

#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/npu_engine.h"
#include "../../include/xdna_b200.h"
#include "capi_internal.h"
#include "toml.h"

namespace xdna {
void read_npy_f32(const std::string &path, std::vector<size_t> &shape, std::vector<float> &data);   // weights.cu
}

namespace {

using xdna::Toml;
thread_local std::string g_npu_err;
void npu_set_err(const std::string &m) { g_npu_err = m; }

// messages of the reference's EngineError variants (api.rs:20-31)
std::string err_load(const std::string &m) { return "load failed: " + m; }
std::string err_unsupported(const std::string &m) { return "unsupported: " + m; }
std::string err_device(const std::string &m) { return "device error: " + m; }

// ------------------------------------------------------------------------------ UTF-8
bool utf8_decode(const std::string &s, std::vector<uint32_t> &cps) {
    cps.clear();
    size_t i = 0;
    while (i < s.size()) {
        const unsigned char c = (unsigned char)s[i];
        uint32_t cp;
        int n;
        if (c < 0x80) { cp = c; n = 0; }
        else if ((c & 0xe0) == 0xc0) { cp = c & 0x1f; n = 1; }
        else if ((c & 0xf0) == 0xe0) { cp = c & 0x0f; n = 2; }
        else if ((c & 0xf8) == 0xf0) { cp = c & 0x07; n = 3; }
        else return false;
        if (i + n >= s.size() + (n ? 0 : 1)) return false;      // truncated sequence
        for (int k = 1; k <= n; k++) {
            const unsigned char d = (unsigned char)s[i + k];
            if ((d & 0xc0) != 0x80) return false;
            cp = (cp << 6) | (d & 0x3f);
        }
        if ((n == 1 && cp < 0x80) || (n == 2 && cp < 0x800) || (n == 3 && cp < 0x10000) || cp > 0x10ffff ||
            (cp >= 0xd800 && cp <= 0xdfff))
            return false;
        cps.push_back(cp);
        i += n + 1;
    }
    return true;
}
void utf8_append(std::string &o, uint32_t cp) {
    if (cp < 0x80) o += (char)cp;
    else if (cp < 0x800) { o += (char)(0xc0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3f)); }
    else if (cp < 0x10000) {
        o += (char)(0xe0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
    } else {
        o += (char)(0xf0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3f));
        o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
    }
}

struct ScenarioCfg {
    std::string kind, name;
    int hidden = 0, ff = 0, n_heads = 0, head_dim = 0, n_layers = 0, max_seq = 0;
    std::string precision = "bf16";
    std::string weights, tokenizer, source, arch, arena;
    std::string pooling = "mean";
    bool normalize = false;
};

ScenarioCfg parse_scenario(const std::string &path) {
    std::ifstream f(path);
    if (!f) throw std::runtime_error("No such file or directory (os error 2)");
    std::stringstream ss;
    ss << f.rdbuf();
    Toml t;
    const std::string e = t.parse(ss.str());
    if (!e.empty()) throw std::runtime_error(e);
    ScenarioCfg c;
    if (!t.has("scenario.kind")) throw std::runtime_error("missing field `kind`");
    if (!t.has("scenario.name")) throw std::runtime_error("missing field `name`");
    c.kind = t.str("scenario.kind");
    c.name = t.str("scenario.name");
    c.hidden = (int)t.integer("model.hidden");
    c.ff = (int)t.integer("model.ff");
    c.n_heads = (int)t.integer("model.n_heads");
    c.head_dim = (int)t.integer("model.head_dim");
    c.n_layers = (int)t.integer("model.n_layers");
    c.max_seq = (int)t.integer("model.max_seq");
    c.precision = t.str("model.precision", "bf16");
    c.weights = t.str("artifacts.weights");
    c.tokenizer = t.str("artifacts.tokenizer");
    c.source = t.str("artifacts.source");
    c.arch = t.str("artifacts.arch");
    c.arena = t.str("artifacts.arena");
    c.pooling = t.str("embeddings.pooling", "mean");
    c.normalize = t.boolean("embeddings.normalize", false);
    return c;
}

// ------------------------------------------------------------------------------ npy
struct Npy {
    std::vector<size_t> shape;
    std::vector<float> data;
};
Npy read_npy(const std::string &path) {
    Npy n;
    xdna::read_npy_f32(path, n.shape, n.data);
    return n;
}

// tensors by name from the legacy npy directory (name + ".npy") or from a baked weight arena
// (the same names, npu-weights/src/arch/bert.rs:121-125 + L{i}/...; bf16 upcast to f32)
struct TensorStore {
    std::string dir;
    XdnaWeightArena *arena = nullptr;
    ~TensorStore() {
        if (arena) xdna_weights_close(arena);
    }
    Npy get(const std::string &name) const {
        if (!arena) return read_npy(dir + "/" + name + ".npy");
        int dt = 0;
        int64_t shape[8];
        const int nd = xdna_weights_info(arena, name.c_str(), &dt, shape, 8);
        if (nd < 0) throw std::runtime_error(std::string("arena: ") + xdna_last_error());
        Npy n;
        size_t count = 1;
        for (int d = 0; d < nd; d++) {
            n.shape.push_back((size_t)shape[d]);
            count *= (size_t)shape[d];
        }
        n.data.resize(count);
        if (xdna_weights_read_f32(arena, name.c_str(), n.data.data(), count) != 0)
            throw std::runtime_error(std::string("arena: ") + xdna_last_error());
        return n;
    }
};

// ------------------------------------------------------------------- WordPiece tokenizer
struct WordPiece {
    std::unordered_map<std::string, int32_t> vocab;
    int32_t unk = -1, cls = -1, sep = -1;
    std::string prefix = "##";
    int max_chars = 100;

    // JSON string body at s[i] (just after the opening quote) -> UTF-8; i moves past the quote
    static std::string json_string(const std::string &s, size_t &i) {
        std::string o;
        while (i < s.size() && s[i] != '"') {
            if (s[i] == '\\' && i + 1 < s.size()) {
                const char e = s[++i];
                if (e == 'u' && i + 4 < s.size()) {
                    uint32_t cp = (uint32_t)std::stoul(s.substr(i + 1, 4), nullptr, 16);
                    i += 4;
                    if (cp >= 0xd800 && cp <= 0xdbff && i + 6 < s.size() && s[i + 1] == '\\' && s[i + 2] == 'u') {
                        const uint32_t lo = (uint32_t)std::stoul(s.substr(i + 3, 4), nullptr, 16);
                        cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                        i += 6;
                    }
                    utf8_append(o, cp);
                } else {
                    o += e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == 'b' ? '\b' : e == 'f' ? '\f' : e;
                }
                i++;
            } else {
                o += s[i++];
            }
        }
        i++;
        return o;
    }

    void load(const std::string &path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("load tokenizer " + path + ": No such file or directory");
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string s = ss.str();
        const bool json = path.size() >= 5 && path.compare(path.size() - 5, 5, ".json") == 0;
        if (json) {
            // "model": { ..., "vocab": { "tok": id, ... } ... }
            size_t m = s.find("\"model\"");
            size_t v = m == std::string::npos ? m : s.find("\"vocab\"", m);
            if (v == std::string::npos) throw std::runtime_error("load tokenizer " + path + ": no model.vocab");
            const size_t ty = s.find("\"type\"", m);
            if (ty != std::string::npos && ty < v && s.find("WordPiece", ty) > s.find(',', ty))
                throw std::runtime_error("load tokenizer " + path + ": not a WordPiece model");
            size_t i = s.find('{', v) + 1;
            while (i < s.size()) {
                while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t' || s[i] == ','))
                    i++;
                if (s[i] == '}') break;
                if (s[i] != '"') throw std::runtime_error("load tokenizer " + path + ": bad vocab entry");
                i++;
                std::string tok = json_string(s, i);
                i = s.find(':', i) + 1;
                char *end = nullptr;
                const long id = std::strtol(s.c_str() + i, &end, 10);
                i = end - s.c_str();
                vocab[tok] = (int32_t)id;
            }
            size_t p = s.find("\"continuing_subword_prefix\"", m);
            if (p != std::string::npos) {
                size_t q = s.find('"', s.find(':', p)) + 1;
                prefix = json_string(s, q);
            }
            p = s.find("\"max_input_chars_per_word\"", m);
            if (p != std::string::npos) max_chars = std::atoi(s.c_str() + s.find(':', p) + 1);
        } else {
            std::istringstream in(s);
            std::string line;
            int32_t id = 0;
            while (std::getline(in, line)) {
                if (!line.empty() && line.back() == '\r') line.pop_back();
                vocab[line] = id++;                      // a repeated token keeps its last id
            }
        }
        auto need = [&](const char *t) -> int32_t {
            auto it = vocab.find(t);
            if (it == vocab.end()) throw std::runtime_error(std::string("load tokenizer ") + path + ": vocabulary has no " + t);
            return it->second;
        };
        unk = need("[UNK]");
        cls = need("[CLS]");
        sep = need("[SEP]");
    }

    static bool is_ws(uint32_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0xa0 || c == 0x3000 || (c >= 0x2000 && c <= 0x200a) || c == 0x202f || c == 0x205f || c == 0x1680; }
    static bool is_ctrl(uint32_t c) { return (c < 0x20 || (c >= 0x7f && c < 0xa0)) && c != '\t' && c != '\n' && c != '\r'; }
    static bool is_punct(uint32_t c) {
        if ((c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126)) return true;
        return c == 0xa1 || c == 0xa7 || c == 0xab || c == 0xb6 || c == 0xb7 || c == 0xbb || c == 0xbf ||
               (c >= 0x2010 && c <= 0x2027) || (c >= 0x2030 && c <= 0x205e) || (c >= 0x3001 && c <= 0x3003) ||
               (c >= 0x3008 && c <= 0x3011);
    }
    static bool is_cjk(uint32_t c) {
        return (c >= 0x4e00 && c <= 0x9fff) || (c >= 0x3400 && c <= 0x4dbf) || (c >= 0x20000 && c <= 0x2a6df) ||
               (c >= 0x2a700 && c <= 0x2b73f) || (c >= 0x2b740 && c <= 0x2b81f) || (c >= 0x2b820 && c <= 0x2ceaf) ||
               (c >= 0xf900 && c <= 0xfaff) || (c >= 0x2f800 && c <= 0x2fa1f);
    }
    // lower case, then accents removed (NFD without combining marks) for Latin-1 letters
    static void lower_strip(uint32_t c, std::vector<uint32_t> &o) {
        if (c >= 'A' && c <= 'Z') { o.push_back(c + 32); return; }
        if (c >= 0x300 && c <= 0x36f) return;                     // combining marks
        if (c >= 0xc0 && c <= 0xff && c != 0xd7 && c != 0xf7) {
            if (c <= 0xde) c += 32;                                // Latin-1 upper -> lower
            // base letter of 0xe0..0xff after dropping the accent (0: no decomposition)
            static const char base[32] = {'a', 'a', 'a', 'a', 'a', 'a', 0,   'c', 'e', 'e', 'e',
                                          'e', 'i', 'i', 'i', 'i', 0,   'n', 'o', 'o', 'o', 'o',
                                          'o', 0,   0,   'u', 'u', 'u', 'u', 'y', 0,   'y'};
            const int k = (int)c - 0xe0;
            if (k >= 0 && k < 32 && base[k]) { o.push_back((uint32_t)base[k]); return; }
            o.push_back(c);
            return;
        }
        o.push_back(c);
    }

    std::vector<int32_t> encode(const std::string &text, int max_len) const {
        std::vector<uint32_t> cps;
        if (!utf8_decode(text, cps)) throw std::runtime_error("text is not valid UTF-8");
        // clean + CJK split + whitespace split + lower/strip + punctuation split
        std::vector<std::vector<uint32_t>> words;
        std::vector<uint32_t> cur;
        auto flush = [&]() { if (!cur.empty()) { words.push_back(cur); cur.clear(); } };
        for (uint32_t c : cps) {
            if (c == 0 || c == 0xfffd || is_ctrl(c)) continue;
            if (is_ws(c)) { flush(); continue; }
            if (is_cjk(c)) { flush(); words.push_back({c}); continue; }
            std::vector<uint32_t> lc;
            lower_strip(c, lc);
            for (uint32_t d : lc) {
                if (is_punct(d)) { flush(); words.push_back({d}); }
                else cur.push_back(d);
            }
        }
        flush();
        std::vector<int32_t> ids{cls};
        for (const auto &w : words) {
            if ((int)w.size() > max_chars) { ids.push_back(unk); continue; }
            std::vector<int32_t> sub;
            size_t start = 0;
            bool bad = false;
            while (start < w.size()) {
                size_t end = w.size();
                int32_t found = -1;
                while (start < end) {
                    std::string piece = start > 0 ? prefix : "";
                    for (size_t k = start; k < end; k++) utf8_append(piece, w[k]);
                    auto it = vocab.find(piece);
                    if (it != vocab.end()) { found = it->second; break; }
                    end--;
                }
                if (found < 0) { bad = true; break; }
                sub.push_back(found);
                start = end;
            }
            if (bad) ids.push_back(unk);
            else ids.insert(ids.end(), sub.begin(), sub.end());
        }
        ids.push_back(sep);
        if ((int)ids.size() > max_len) ids.resize(max_len);        // frontend.rs:31-33
        return ids;
    }
};

}  // namespace

// --------------------------------------------------------------------------- model handle
namespace xdna {
struct AsrState;   // asr.cu: the Whisper pipeline behind npu_transcribe
AsrState *asr_load(XdnaDevice *dev, const std::string &wdir, const std::string &tokenizer, int n_layers);
void asr_free(AsrState *a);
std::string asr_transcribe(AsrState *a, const int16_t *pcm, size_t n);
}  // namespace xdna

struct NpuModel {
    ScenarioCfg cfg;
    XdnaDevice *dev = nullptr;
    XdnaBert *bert = nullptr;
    xdna::AsrState *asr = nullptr;
    WordPiece tok;
    ~NpuModel() {
        if (bert) xdna_bert_free(bert);
        if (asr) xdna::asr_free(asr);
        if (dev) xdna_device_close(dev);
    }
};

namespace {

NpuModel *load_embed(const ScenarioCfg &c, const std::string &path, int ordinal) {
    if (c.hidden != 768 || c.ff != 3072 || c.n_heads != 12 || c.head_dim != 64)
        throw std::runtime_error(err_unsupported("embedding models with hidden 768, ff 3072, 12 heads of 64 (BERT-base)"));
    if (c.n_layers < 1 || c.max_seq < 1) throw std::runtime_error(err_load("scenario " + path + ": bad model sizes"));
    std::unique_ptr<NpuModel> m(new NpuModel());
    m->cfg = c;
    char cwd[4096];
    const std::string root = getcwd(cwd, sizeof cwd) ? std::string(cwd) : std::string(".");
    m->tok.load(root + "/" + c.tokenizer);
    // weights: a baked arena when artifacts.source is set (BertWeights::load_for,
    // bert/weights.rs:41-53), else the legacy npy directory artifacts.weights
    TensorStore store;
    std::string wdir = root + "/" + c.weights;
    if (!c.source.empty()) {
        if (c.arch.empty())
            throw std::runtime_error(err_load("artifacts.source is set but artifacts.arch is empty (need "
                                              "bert|esm|vit|opt|whisper|fastconformer|gigaam)"));
        if (c.source.rfind("hf:", 0) != 0 && c.source.rfind("path:", 0) != 0)
            throw std::runtime_error(err_load("artifacts.source \"" + c.source + "\": expected hf:<repo>[@rev] or path:/abs"));
        if (c.arena.empty())
            throw std::runtime_error(err_unsupported("baking a weight arena from artifacts.source (npu-weights bake); "
                                                     "set artifacts.arena to a baked arena"));
        wdir = c.arena[0] == '/' ? c.arena : root + "/" + c.arena;
        store.arena = xdna_weights_open(wdir.c_str(), c.arch.c_str());
        if (!store.arena) throw std::runtime_error(err_load(xdna_last_error()));
    } else {
        store.dir = wdir;
    }
    std::map<std::string, Npy> emb;
    for (const char *k : {"word_emb", "pos_emb", "type_emb", "emb_ln_w", "emb_ln_b"})
        emb[k] = store.get(std::string("emb/") + k);
    static const char *names[] = {"q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "attn_out_w", "attn_out_b",
                                  "attn_ln_w", "attn_ln_b", "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b", "out_ln_w",
                                  "out_ln_b"};
    std::vector<std::map<std::string, Npy>> layers(c.n_layers);
    for (int l = 0; l < c.n_layers; l++)
        for (const char *k : names) layers[l][k] = store.get("L" + std::to_string(l) + "/" + k);
    const Npy &we = emb["word_emb"], &pe = emb["pos_emb"];
    if (we.shape.size() != 2 || we.shape[1] != 768 || pe.shape.size() != 2 || pe.shape[1] != 768)
        throw std::runtime_error(err_load("bert weights load " + wdir + ": embedding tables must be [n, 768]"));
    for (const auto &kv : m->tok.vocab)
        if (kv.second < 0 || (size_t)kv.second >= we.shape[0])
            throw std::runtime_error(err_load("tokenizer id " + std::to_string(kv.second) + " beyond the embedding table"));
    XdnaBertConfig bc{};
    bc.n_layers = c.n_layers;
    bc.d_model = 768;
    bc.n_heads = 12;
    bc.ffn = 3072;
    bc.vocab = (int)we.shape[0];
    bc.max_pos = (int)pe.shape[0];
    bc.eps = 1e-12f;                                  // BERT LayerNorm eps (frontend.rs:13)
    bc.pooling = (c.pooling == "cls" ? 0 : 1) + (c.normalize ? 0 : 2);   // head.rs:14-17
    std::vector<XdnaBertLayer> ly(c.n_layers);
    for (int l = 0; l < c.n_layers; l++) {
        auto &L = layers[l];
        ly[l] = XdnaBertLayer{L["q_w"].data.data(), L["q_b"].data.data(), L["k_w"].data.data(),
                              L["k_b"].data.data(), L["v_w"].data.data(), L["v_b"].data.data(),
                              L["attn_out_w"].data.data(), L["attn_out_b"].data.data(),
                              L["attn_ln_w"].data.data(), L["attn_ln_b"].data.data(), L["ffn1_w"].data.data(),
                              L["ffn1_b"].data.data(), L["ffn2_w"].data.data(), L["ffn2_b"].data.data(),
                              L["out_ln_w"].data.data(), L["out_ln_b"].data.data()};
    }
    XdnaBertWeights bw{we.data.data(), pe.data.data(), emb["type_emb"].data.data(), emb["emb_ln_w"].data.data(),
                       emb["emb_ln_b"].data.data(), ly.data()};
    m->dev = xdna_device_open(ordinal);
    if (!m->dev) throw std::runtime_error(err_device(xdna_last_error()));
    const int max_len = std::min(c.max_seq, bc.max_pos);
    m->cfg.max_seq = max_len;
    m->bert = xdna_bert_create(m->dev, &bc, &bw, max_len, 1);
    if (!m->bert) throw std::runtime_error(err_load(xdna_last_error()));
    return m.release();
}

// ASR scenarios: Whisper-small (hidden 768, 12 heads of 64, ff 3072) from the npy layout of
// artifacts.weights; the tokenizer is artifacts.tokenizer, else tokenizer.json beside the weights
NpuModel *load_asr(const ScenarioCfg &c, const std::string &path, int ordinal) {
    if (c.name.find("whisper") == std::string::npos)
        throw std::runtime_error(err_unsupported("ASR model \"" + c.name + "\": only Whisper scenarios are wired "
                                                 "behind npu_transcribe"));
    if (c.hidden != 768 || c.ff != 3072 || c.n_heads != 12 || c.head_dim != 64)
        throw std::runtime_error(err_unsupported("ASR models with hidden 768, ff 3072, 12 heads of 64 (Whisper-small)"));
    if (!c.source.empty())
        throw std::runtime_error(err_unsupported("artifacts.source (weight arenas); give the npy directory in artifacts.weights"));
    std::unique_ptr<NpuModel> m(new NpuModel());
    m->cfg = c;
    char cwd[4096];
    const std::string root = getcwd(cwd, sizeof cwd) ? std::string(cwd) : std::string(".");
    const std::string wdir = root + "/" + c.weights;
    const std::string tok = c.tokenizer.empty() ? wdir + "/tokenizer.json" : root + "/" + c.tokenizer;
    struct stat st;
    if (c.weights.empty() || stat(wdir.c_str(), &st) != 0 || !S_ISDIR(st.st_mode))
        throw std::runtime_error(err_load("asr weights load " + wdir + ": No such file or directory"));
    m->dev = xdna_device_open(ordinal);
    if (!m->dev) throw std::runtime_error(err_device(xdna_last_error()));
    try {
        m->asr = xdna::asr_load(m->dev, wdir, tok, c.n_layers);
    } catch (const std::exception &e) {
        throw std::runtime_error(err_load("asr weights load " + wdir + ": " + e.what()));
    }
    (void)path;
    return m.release();
}

}  // namespace

void npu_set_last_error(const std::string &msg) { npu_set_err(msg); }

// npu_model_load on a given CUDA device (the control plane loads one replica per GPU)
NpuModel *npu_model_load_on(const char *scenario_path, int ordinal) {
    try {
        if (!scenario_path) { npu_set_err("scenario_path is null"); return nullptr; }
        const std::string path(scenario_path);
        std::vector<uint32_t> cps;
        if (!utf8_decode(path, cps)) { npu_set_err("scenario_path is not valid UTF-8"); return nullptr; }
        ScenarioCfg c;
        try {
            c = parse_scenario(path);
        } catch (const std::exception &e) {
            npu_set_err(err_load("scenario " + path + ": " + e.what()));
            return nullptr;
        }
        if (c.kind == "embeddings") return load_embed(c, path, ordinal);
        if (c.kind == "asr") return load_asr(c, path, ordinal);
        npu_set_err(err_load("unknown scenario kind \"" + c.kind + "\""));
        return nullptr;
    } catch (const std::exception &e) {
        npu_set_err(e.what());
        return nullptr;
    } catch (...) {
        npu_set_err("panic in npu_model_load");
        return nullptr;
    }
}

extern "C" {

int npu_available(void) {
    try {
        return xdna_device_count() > 0 ? 1 : 0;
    } catch (...) {
        return 0;
    }
}

NpuModel *npu_model_load(const char *scenario_path) { return npu_model_load_on(scenario_path, 0); }

int npu_model_kind(const NpuModel *m) {
    if (!m) { npu_set_err("model is null"); return -1; }
    return m->cfg.kind == "asr" ? 0 : 1;
}

char *npu_transcribe(NpuModel *m, const int16_t *pcm, uintptr_t n, uint32_t sample_rate) {
    if (!m) { npu_set_err("model is null"); return nullptr; }
    if (!pcm && n != 0) { npu_set_err("pcm is null"); return nullptr; }
    if (sample_rate != 16000) {
        npu_set_err(err_unsupported("sample_rate " + std::to_string(sample_rate) + " (need 16000)"));
        return nullptr;
    }
    if (!m->asr) {
        npu_set_err("wrong model kind: wanted asr, got embed");
        return nullptr;
    }
    try {
        const std::string text = xdna::asr_transcribe(m->asr, pcm, (size_t)n);
        if (text.find('\0') != std::string::npos) {
            npu_set_err("transcript contained a NUL byte");
            return nullptr;
        }
        char *r = static_cast<char *>(std::malloc(text.size() + 1));
        if (!r) { npu_set_err("out of host memory"); return nullptr; }
        std::memcpy(r, text.c_str(), text.size() + 1);
        return r;
    } catch (const std::exception &e) {
        npu_set_err(err_device(e.what()));
        return nullptr;
    } catch (...) {
        npu_set_err("panic in npu_transcribe");
        return nullptr;
    }
}

int npu_embed(NpuModel *m, const char *text, float *out, uintptr_t out_cap) {
    try {
        if (!m) { npu_set_err("model is null"); return -1; }
        if (m->cfg.kind != "embeddings") { npu_set_err("model is not an embedder"); return -1; }
        const int dim = m->cfg.hidden;
        if (!out || out_cap == 0) return dim;
        if (!text) { npu_set_err("text is null"); return -1; }
        std::vector<int32_t> ids;
        try {
            ids = m->tok.encode(text, m->cfg.max_seq);
        } catch (const std::exception &e) {
            npu_set_err(e.what());
            return -1;
        }
        const int32_t len = (int32_t)ids.size();
        std::vector<float> v(dim);
        if (xdna_bert_embed(m->bert, ids.data(), &len, 1, v.data()) != 0) {
            npu_set_err(err_device(xdna_last_error()));
            return -1;
        }
        std::memcpy(out, v.data(), sizeof(float) * std::min<uintptr_t>((uintptr_t)dim, out_cap));
        return dim;
    } catch (const std::exception &e) {
        npu_set_err(e.what());
        return -1;
    } catch (...) {
        npu_set_err("panic in npu_embed");
        return -1;
    }
}

void npu_string_free(char *s) { std::free(s); }

void npu_model_free(NpuModel *m) {
    try {
        delete m;
    } catch (...) {
    }
}

const char *npu_last_error(void) { return g_npu_err.c_str(); }

// WordPiece front end on its own (host only): the ids npu_embed feeds the encoder for `text`.
int xdna_wordpiece_encode(const char *tokenizer_path, const char *text, int max_len, int32_t *ids, int cap) {
    try {
        if (!tokenizer_path || !text || !ids) { npu_set_err("xdna_wordpiece_encode: null pointer"); return -1; }
        WordPiece wp;
        wp.load(tokenizer_path);
        const std::vector<int32_t> v = wp.encode(text, max_len);
        std::memcpy(ids, v.data(), sizeof(int32_t) * std::min<size_t>(v.size(), (size_t)std::max(cap, 0)));
        return (int)v.size();
    } catch (const std::exception &e) {
        npu_set_err(e.what());
        return -1;
    }
}

}  // extern "C"
