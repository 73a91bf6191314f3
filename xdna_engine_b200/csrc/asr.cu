// asr.cu -- the Whisper ASR scenario behind npu_transcribe: what WhisperAsr::transcribe does
// (rust/npu-engine/src/asr/whisper.rs:682-745), with every stage on the GPU except the control
// logic and the detokenizer:
//
//   pcm i16 -> / 32768, zero-padded or truncated to 480,000 samples -> log-mel [80][3000]
//   (xdna_log_mel) -> encoder [1500][768] (xdna_whisper_encode) -> language detection: one
//   decoder step on <|startoftranscript|>, argmax restricted to the language-tag block
//   50259..50357 (pick_lang, whisper.rs:312-322) -> greedy decode of up to 200 tokens after
//   [SOT, lang, <|transcribe|>, <|notimestamps|>], stopping at <|endoftext|> (whisper.rs:426-465;
//   full-vocabulary argmax, first maximum) -> detokenize with special tokens skipped, trimmed
//   (whisper.rs:671-679).
//
// The detokenizer restates what the HuggingFace `tokenizers` library does with a Whisper
// tokenizer.json (BPE model + ByteLevel decoder): ids -> token strings (added tokens first,
// then the BPE vocabulary; unknown ids dropped), special added tokens dropped when asked, the
// strings' characters mapped back to bytes through the inverse of GPT-2's byte-to-unicode
// table (a token with a character outside the table keeps its own UTF-8 bytes), and the bytes
// decoded as UTF-8 with invalid sequences replaced by U+FFFD.
//
// Weights: the reference's npy layout under artifacts.weights (npu-whisper/src/weights.rs:42-80,
// npu-engine/src/asr/whisper_decoder.rs:113-160): L{i}/{ln1,ln2,q,k,v,out,fc1,fc2}.{weight,bias}
// ([in, out] linear weights), conv/{conv1,conv2}.{weight,bias} + conv/embed_positions,
// refs/ln_post.{weight,bias}; whisper_decoder/{embed_tokens, embed_positions, proj_out.weight,
// ln_post.*} and whisper_decoder/L{i}/{ln_self, q, k, v, out, ln_cross, cross_q, cross_k,
// cross_v, cross_out, ln_final, fc1, fc2}.{weight,bias}; tokenizer.json beside them.
#include <sys/stat.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/xdna_b200.h"
#include "json.h"

namespace xdna {
void set_last_error_message(const std::string &m);
void read_npy_f32(const std::string &path, std::vector<size_t> &shape, std::vector<float> &data);

// ------------------------------------------------------------------------ byte-level BPE decode
struct BpeDecoder {
    std::vector<std::string> id_tok;      // id -> token string (UTF-8); empty + !known = unknown id
    std::vector<uint8_t> known, special;
    int byte_of[512];                     // code point (< 512) -> byte, or -1

    BpeDecoder() {
        // GPT-2's byte-to-unicode table: printable bytes map to themselves, the other 68 bytes to
        // U+0100.. in increasing byte order
        std::fill(byte_of, byte_of + 512, -1);
        int n = 0;
        for (int b = 0; b < 256; b++) {
            const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
            byte_of[printable ? b : 256 + n++] = b;
        }
    }

    void put(int id, const std::string &tok, bool is_special) {
        if (id < 0) return;
        if ((size_t)id >= id_tok.size()) {
            id_tok.resize(id + 1);
            known.resize(id + 1, 0);
            special.resize(id + 1, 0);
        }
        id_tok[id] = tok;
        known[id] = 1;
        special[id] = is_special ? 1 : 0;
    }

    void load(const std::string &path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("read " + path + ": No such file or directory");
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string s = ss.str();
        json::JsonParser jp{s.data(), s.data() + s.size(), "tokenizer.json"};
        const json::Json root = jp.value();
        auto model = root.obj.find("model");
        if (model == root.obj.end()) throw std::runtime_error(path + ": no \"model\"");
        auto vocab = model->second.obj.find("vocab");
        if (vocab == model->second.obj.end() || vocab->second.kind != json::Json::Obj)
            throw std::runtime_error(path + ": the model has no vocabulary object");
        for (const auto &kv : vocab->second.obj) put((int)kv.second.num, kv.first, false);
        auto added = root.obj.find("added_tokens");
        if (added != root.obj.end())
            for (const auto &t : added->second.arr) {
                auto id = t.obj.find("id"), content = t.obj.find("content"), sp = t.obj.find("special");
                if (id == t.obj.end() || content == t.obj.end()) continue;
                put((int)id->second.num, content->second.str, sp != t.obj.end() && sp->second.b);
            }
    }

    static bool next_cp(const std::string &s, size_t &i, uint32_t &cp) {
        const unsigned char c = (unsigned char)s[i];
        int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
        if (n == 0 || i + n > s.size()) { i++; return false; }
        cp = n == 1 ? c : n == 2 ? (c & 0x1f) : n == 3 ? (c & 0x0f) : (c & 0x07);
        for (int k = 1; k < n; k++) cp = (cp << 6) | ((unsigned char)s[i + k] & 0x3f);
        i += n;
        return true;
    }
    static void put_utf8(std::string &o, uint32_t cp) {
        if (cp < 0x80) o += (char)cp;
        else if (cp < 0x800) { o += (char)(0xc0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3f)); }
        else if (cp < 0x10000) {
            o += (char)(0xe0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
        } else {
            o += (char)(0xf0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3f));
            o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
        }
    }
    // bytes -> UTF-8 text, each maximal invalid subsequence replaced by U+FFFD (the rule of
    // Rust's String::from_utf8_lossy)
    static std::string lossy(const std::string &b) {
        std::string o;
        size_t i = 0;
        while (i < b.size()) {
            const unsigned char c = (unsigned char)b[i];
            int n = 0;
            uint32_t lo = 0x80, hi = 0xbf;
            if (c < 0x80) { o += (char)c; i++; continue; }
            if (c >= 0xc2 && c <= 0xdf) n = 2;
            else if (c >= 0xe0 && c <= 0xef) { n = 3; if (c == 0xe0) lo = 0xa0; if (c == 0xed) hi = 0x9f; }
            else if (c >= 0xf0 && c <= 0xf4) { n = 4; if (c == 0xf0) lo = 0x90; if (c == 0xf4) hi = 0x8f; }
            if (n == 0) { put_utf8(o, 0xfffd); i++; continue; }
            size_t k = 1;
            for (; k < (size_t)n && i + k < b.size(); k++) {
                const unsigned char d = (unsigned char)b[i + k];
                const uint32_t l2 = k == 1 ? lo : 0x80, h2 = k == 1 ? hi : 0xbf;
                if (d < l2 || d > h2) break;
            }
            if (k == (size_t)n) { o.append(b, i, n); i += n; }
            else { put_utf8(o, 0xfffd); i += k; }
        }
        return o;
    }

    std::string decode(const int64_t *ids, size_t n, bool skip_special) const {
        std::string bytes;
        for (size_t j = 0; j < n; j++) {
            const int64_t id = ids[j];
            if (id < 0 || (size_t)id >= id_tok.size() || !known[id]) continue;
            if (skip_special && special[id]) continue;
            // a token whose characters all come from the byte table becomes those bytes; any other
            // token is kept as its own UTF-8 bytes, whole
            const std::string &t = id_tok[id];
            std::string tb;
            bool mapped = true;
            size_t i = 0;
            while (i < t.size() && mapped) {
                uint32_t cp = 0;
                if (!next_cp(t, i, cp) || cp >= 512 || byte_of[cp] < 0) mapped = false;
                else tb += (char)byte_of[cp];
            }
            bytes += mapped ? tb : t;
        }
        return lossy(bytes);
    }
};

// ------------------------------------------------------------------------------- the scenario
struct AsrState {
    XdnaLogMel *lm = nullptr;
    XdnaWhisperEnc *enc = nullptr;
    XdnaWhisperDec *dec = nullptr;
    BpeDecoder tok;
    int vocab = 0;
    ~AsrState() {
        if (dec) xdna_whisper_dec_free(dec);
        if (enc) xdna_whisper_enc_free(enc);
        if (lm) xdna_log_mel_free(lm);
    }
};

namespace {

constexpr int64_t kSot = 50258, kEot = 50257, kTranscribe = 50359, kNoTimestamps = 50363;
constexpr int64_t kLangLo = 50259, kLangHi = 50357;
constexpr int kMaxDecode = 200;

struct NpyStore {
    std::string dir;
    std::vector<std::vector<float>> keep;
    const float *get(const std::string &name, const std::vector<size_t> &expect) {
        std::vector<size_t> shape;
        keep.emplace_back();
        read_npy_f32(dir + "/" + name + ".npy", shape, keep.back());
        if (shape != expect) {
            std::string a, b;
            for (size_t v : shape) a += std::to_string(v) + ",";
            for (size_t v : expect) b += std::to_string(v) + ",";
            throw std::runtime_error(dir + "/" + name + ".npy has shape [" + a + "], expected [" + b + "]");
        }
        return keep.back().data();
    }
};

// Rust's str::trim: strip leading and trailing code points with the Unicode White_Space property
bool white_space(uint32_t c) {
    return (c >= 0x09 && c <= 0x0d) || c == 0x20 || c == 0x85 || c == 0xa0 || c == 0x1680 || (c >= 0x2000 && c <= 0x200a) ||
           c == 0x2028 || c == 0x2029 || c == 0x202f || c == 0x205f || c == 0x3000;
}
std::string trim_unicode(const std::string &t) {
    std::vector<std::pair<size_t, uint32_t>> cps;     // (byte offset, code point); t is valid UTF-8
    for (size_t i = 0; i < t.size();) {
        const size_t at = i;
        uint32_t cp = 0;
        if (!BpeDecoder::next_cp(t, i, cp)) cp = 0xfffd;
        cps.emplace_back(at, cp);
    }
    size_t b = 0, e = cps.size();
    while (b < e && white_space(cps[b].second)) b++;
    while (e > b && white_space(cps[e - 1].second)) e--;
    if (b == e) return "";
    const size_t end = e < cps.size() ? cps[e].first : t.size();
    return t.substr(cps[b].first, end - cps[b].first);
}

bool is_dir(const std::string &p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

}  // namespace

AsrState *asr_load(XdnaDevice *dev, const std::string &wdir, const std::string &tokenizer, int n_layers) {
    std::unique_ptr<AsrState> a(new AsrState());
    a->tok.load(tokenizer);
    constexpr size_t D = 768, F = 3072;
    // ---- encoder
    NpyStore e{wdir};
    int ne = 0;
    while (is_dir(wdir + "/L" + std::to_string(ne))) ne++;
    if (ne == 0) throw std::runtime_error(wdir + ": no encoder blocks (L0/ missing)");
    if (n_layers > 0 && ne != n_layers)
        throw std::runtime_error(wdir + ": " + std::to_string(ne) + " encoder blocks, the scenario says " +
                                 std::to_string(n_layers));
    std::vector<XdnaWhisperEncLayer> el(ne);
    for (int l = 0; l < ne; l++) {
        const std::string p = "L" + std::to_string(l) + "/";
        XdnaWhisperEncLayer &y = el[l];
        y.ln1_w = e.get(p + "ln1.weight", {D});
        y.ln1_b = e.get(p + "ln1.bias", {D});
        y.q_w = e.get(p + "q.weight", {D, D});
        y.q_b = e.get(p + "q.bias", {D});
        y.k_w = e.get(p + "k.weight", {D, D});
        y.k_b = e.get(p + "k.bias", {D});
        y.v_w = e.get(p + "v.weight", {D, D});
        y.v_b = e.get(p + "v.bias", {D});
        y.out_w = e.get(p + "out.weight", {D, D});
        y.out_b = e.get(p + "out.bias", {D});
        y.ln2_w = e.get(p + "ln2.weight", {D});
        y.ln2_b = e.get(p + "ln2.bias", {D});
        y.fc1_w = e.get(p + "fc1.weight", {D, F});
        y.fc1_b = e.get(p + "fc1.bias", {F});
        y.fc2_w = e.get(p + "fc2.weight", {F, D});
        y.fc2_b = e.get(p + "fc2.bias", {D});
    }
    XdnaWhisperEncWeights ew{};
    ew.conv1_w = e.get("conv/conv1.weight", {D, 80, 3});
    ew.conv1_b = e.get("conv/conv1.bias", {D});
    ew.conv2_w = e.get("conv/conv2.weight", {D, D, 3});
    ew.conv2_b = e.get("conv/conv2.bias", {D});
    ew.embed_positions = e.get("conv/embed_positions", {1500, D});
    ew.ln_post_w = e.get("refs/ln_post.weight", {D});
    ew.ln_post_b = e.get("refs/ln_post.bias", {D});
    ew.layers = el.data();
    XdnaWhisperEncConfig ec{ne, (int)D, 12, (int)F, 80, 3000, 1500, 1e-5f};
    a->enc = xdna_whisper_enc_create(dev, &ec, &ew, 1);
    if (!a->enc) throw std::runtime_error(std::string("encoder: ") + xdna_last_error());
    e.keep.clear();
    // ---- decoder
    const std::string ddir = wdir + "/whisper_decoder";
    NpyStore d{ddir};
    std::vector<size_t> sh;
    std::vector<float> probe;
    read_npy_f32(ddir + "/embed_tokens.npy", sh, probe);
    if (sh.size() != 2 || sh[1] != D) throw std::runtime_error(ddir + "/embed_tokens.npy must be [vocab, 768]");
    const size_t V = sh[0];
    if (V <= (size_t)kNoTimestamps) throw std::runtime_error("decoder vocabulary too small for Whisper's special tokens");
    probe.clear();
    read_npy_f32(ddir + "/embed_positions.npy", sh, probe);
    if (sh.size() != 2 || sh[1] != D || sh[0] < 4 + kMaxDecode)
        throw std::runtime_error(ddir + "/embed_positions.npy must be [>= 204, 768]");
    const size_t T = sh[0];
    probe.clear();
    int nd = 0;
    while (is_dir(ddir + "/L" + std::to_string(nd))) nd++;
    if (nd == 0) throw std::runtime_error(ddir + ": no decoder layers");
    std::vector<XdnaWhisperDecLayer> dl(nd);
    for (int l = 0; l < nd; l++) {
        const std::string p = "L" + std::to_string(l) + "/";
        XdnaWhisperDecLayer &y = dl[l];
        auto lin = [&](const char *n, const float *&w, const float *&b) {
            w = d.get(p + n + ".weight", {D, D});
            b = d.get(p + n + ".bias", {D});
        };
        y.ln_self_w = d.get(p + "ln_self.weight", {D});
        y.ln_self_b = d.get(p + "ln_self.bias", {D});
        lin("q", y.q_w, y.q_b);
        lin("k", y.k_w, y.k_b);
        lin("v", y.v_w, y.v_b);
        lin("out", y.out_w, y.out_b);
        y.ln_cross_w = d.get(p + "ln_cross.weight", {D});
        y.ln_cross_b = d.get(p + "ln_cross.bias", {D});
        lin("cross_q", y.cross_q_w, y.cross_q_b);
        lin("cross_k", y.cross_k_w, y.cross_k_b);
        lin("cross_v", y.cross_v_w, y.cross_v_b);
        lin("cross_out", y.cross_out_w, y.cross_out_b);
        y.ln_final_w = d.get(p + "ln_final.weight", {D});
        y.ln_final_b = d.get(p + "ln_final.bias", {D});
        y.fc1_w = d.get(p + "fc1.weight", {D, F});
        y.fc1_b = d.get(p + "fc1.bias", {F});
        y.fc2_w = d.get(p + "fc2.weight", {F, D});
        y.fc2_b = d.get(p + "fc2.bias", {D});
    }
    XdnaWhisperDecWeights dw{};
    dw.embed_tokens = d.get("embed_tokens", {V, D});
    dw.embed_positions = d.get("embed_positions", {T, D});
    dw.proj_out = d.get("proj_out.weight", {D, V});
    dw.ln_post_w = d.get("ln_post.weight", {D});
    dw.ln_post_b = d.get("ln_post.bias", {D});
    dw.layers = dl.data();
    XdnaWhisperDecConfig dc{nd, (int)D, 12, (int)F, (int)V, (int)T, 1500};
    a->dec = xdna_whisper_dec_create(dev, &dc, &dw, 1);
    if (!a->dec) throw std::runtime_error(std::string("decoder: ") + xdna_last_error());
    a->vocab = (int)V;
    a->lm = xdna_log_mel_create(dev);
    if (!a->lm) throw std::runtime_error(std::string("log-mel: ") + xdna_last_error());
    return a.release();
}

void asr_free(AsrState *a) { delete a; }

// the transcript, or throws with the failing stage
std::string asr_transcribe(AsrState *a, const int16_t *pcm, size_t n) {
    std::vector<float> mel(80 * 3000), encs((size_t)1500 * 768);
    if (xdna_log_mel(a->lm, pcm, n, mel.data()) != 0) throw std::runtime_error(xdna_last_error());
    if (xdna_whisper_encode(a->enc, mel.data(), 1, encs.data()) != 0) throw std::runtime_error(xdna_last_error());
    // language detection: one step on <|startoftranscript|>, argmax over the language block
    std::vector<float> logits(a->vocab);
    int64_t tok0 = 0;
    if (xdna_whisper_dec_generate(a->dec, encs.data(), 1, &kSot, 1, 1, &tok0, logits.data()) != 0)
        throw std::runtime_error(xdna_last_error());
    int64_t lang = kLangLo;
    for (int64_t i = kLangLo; i <= kLangHi; i++)
        if (logits[i] > logits[lang]) lang = i;
    // greedy decode after the prompt, up to the first <|endoftext|>
    const int64_t prompt[4] = {kSot, lang, kTranscribe, kNoTimestamps};
    std::vector<int64_t> out(kMaxDecode);
    if (xdna_whisper_dec_generate(a->dec, encs.data(), 1, prompt, 4, kMaxDecode, out.data(), nullptr) != 0)
        throw std::runtime_error(xdna_last_error());
    std::vector<int64_t> ids(prompt, prompt + 4);
    for (int64_t t : out) {
        if (t == kEot) break;
        ids.push_back(t);
    }
    return trim_unicode(a->tok.decode(ids.data(), ids.size(), true));
}

}  // namespace xdna

extern "C" int xdna_bpe_decode(const char *tokenizer_path, const int64_t *ids, size_t n, int skip_special, char *out,
                               size_t cap) {
    try {
        if (!tokenizer_path || (!ids && n)) { xdna::set_last_error_message("xdna_bpe_decode: null pointer"); return -1; }
        xdna::BpeDecoder d;
        d.load(tokenizer_path);
        const std::string s = d.decode(ids, n, skip_special != 0);
        if (out && cap) {
            const size_t k = std::min(cap - 1, s.size());
            std::memcpy(out, s.data(), k);
            out[k] = 0;
        }
        return (int)s.size();
    } catch (const std::exception &e) {
        xdna::set_last_error_message(std::string("xdna_bpe_decode: ") + e.what());
        return -1;
    }
}
