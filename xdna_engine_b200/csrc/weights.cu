// weights.cu -- weight stores: the baked safetensors "arena" and the legacy npy directory, and
// the opt-125m loader over either.
//
// * Arena (rust/npu-weights/src/arena.rs:13-80): one safetensors file -- 8-byte little-endian
//   header length, a JSON header mapping each tensor name to {dtype, shape, data_offsets} plus
//   "__metadata__" {format_version, arch, source_ref, source_fingerprint}, then the tensor
//   bytes.  Opening checks the arch against the caller's and format_version == 1 (arena.rs:51-56,
//   lib.rs:11), with the reference's messages.  Tensors are BF16 or F32 little-endian; reads
//   upcast bf16 to f32 (tensor_f32) or hand out the raw bf16 bits (tensor_bf16, arena.rs:86-100).
//   The file is memory-mapped and never copied whole.
// * npy directory: the same names with ".npy" appended (the arena's names equal the npy paths
//   relative to the artifact directory, arch/opt.rs:4-6), f32 little-endian C order.
// * xdna_opt_load: Opt::load (rust/npu-whisper/src/bin/opt125m_decode.rs:155-180) from either
//   store, names per arch/opt.rs:7-16 (embed_tokens, embed_positions, ln_final.*, lm_head.weight
//   [d, vocab], L{i}/{q,k,v,out,fc1,fc2}.{weight [in, out], bias}, L{i}/ln_{self,ffn}.*); the
//   shapes give the config.  The decoder's LM head is the tied embedding, so lm_head.weight must
//   equal embed_tokens transposed (true of OPT checkpoints; arch/opt.rs:19-22).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"
#include "json.h"

namespace xdna {
void set_last_error_message(const std::string &m);
}
using xdna::set_last_error_message;

using xdna::json::Json;
using xdna::json::JsonParser;

namespace {

uint64_t as_u64(const Json &j, const char *what) {
    if (j.kind != Json::Num || j.num < 0 || j.num != (double)(uint64_t)j.num)
        throw std::runtime_error(std::string("safetensors header: ") + what + " is not a non-negative integer");
    return (uint64_t)j.num;
}

float bf16_to_f32(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

}  // namespace

namespace xdna {
// f32 npy (little-endian, C order) -> shape + data; throws with the path on any problem.
void read_npy_f32(const std::string &path, std::vector<size_t> &shape, std::vector<float> &data) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("read " + path + ": No such file or directory");
    char magic[8];
    f.read(magic, 8);
    if (!f || std::memcmp(magic, "\x93NUMPY", 6) != 0) throw std::runtime_error("read " + path + ": not an npy file");
    uint32_t hlen = 0;
    unsigned char b[4] = {0, 0, 0, 0};
    f.read(reinterpret_cast<char *>(b), magic[6] == 1 ? 2 : 4);
    hlen = b[0] | (b[1] << 8) | (b[2] << 16) | ((uint32_t)b[3] << 24);
    std::string h(hlen, '\0');
    f.read(&h[0], hlen);
    if (h.find("'descr': '<f4'") == std::string::npos)
        throw std::runtime_error("read " + path + ": expected little-endian f32 data");
    if (h.find("'fortran_order': False") == std::string::npos)
        throw std::runtime_error("read " + path + ": Fortran order is not supported");
    const size_t a = h.find("'shape': ("), e = h.find(')', a);
    if (a == std::string::npos || e == std::string::npos) throw std::runtime_error("read " + path + ": bad header");
    shape.clear();
    size_t count = 1;
    const std::string dims = h.substr(a + 10, e - a - 10);
    size_t i = 0;
    while (i < dims.size()) {
        while (i < dims.size() && (dims[i] == ' ' || dims[i] == ',')) i++;
        if (i >= dims.size()) break;
        size_t j = i;
        while (j < dims.size() && dims[j] >= '0' && dims[j] <= '9') j++;
        if (j == i) throw std::runtime_error("read " + path + ": bad shape");
        shape.push_back(std::stoul(dims.substr(i, j - i)));
        count *= shape.back();
        i = j;
    }
    data.resize(count);
    f.read(reinterpret_cast<char *>(data.data()), count * 4);
    if (!f) throw std::runtime_error("read " + path + ": file shorter than its shape");
}
}  // namespace xdna

struct XdnaWeightArena {
    struct Tensor {
        int dtype;                   // 0 F32, 1 BF16
        std::vector<int64_t> shape;
        size_t begin, end;           // byte range in the data section
    };
    void *map = MAP_FAILED;
    size_t map_bytes = 0;
    const uint8_t *data = nullptr;   // start of the data section
    std::map<std::string, Tensor> tensors;
    std::vector<std::string> names;  // sorted (the header's map order)
    std::map<std::string, std::string> meta;
    ~XdnaWeightArena() {
        if (map != MAP_FAILED) munmap(map, map_bytes);
    }
    const Tensor &get(const std::string &name) const {
        auto it = tensors.find(name);
        if (it == tensors.end()) throw std::runtime_error("tensor \"" + name + "\" not in the arena");
        return it->second;
    }
    size_t count(const Tensor &t) const { return (t.end - t.begin) / (t.dtype ? 2 : 4); }
    void read_f32(const Tensor &t, float *out) const {
        const uint8_t *s = data + t.begin;
        const size_t n = count(t);
        if (t.dtype == 0) std::memcpy(out, s, n * 4);
        else
            for (size_t i = 0; i < n; i++) {
                uint16_t h;
                std::memcpy(&h, s + 2 * i, 2);
                out[i] = bf16_to_f32(h);
            }
    }
};

namespace {

XdnaWeightArena *open_arena(const std::string &path, const char *expect_arch) {
    std::unique_ptr<XdnaWeightArena> a(new XdnaWeightArena());
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("open " + path + ": No such file or directory");
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
        ::close(fd);
        throw std::runtime_error(path + ": not a safetensors file (shorter than its header length)");
    }
    a->map_bytes = (size_t)st.st_size;
    a->map = mmap(nullptr, a->map_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (a->map == MAP_FAILED) throw std::runtime_error("mmap " + path + " failed");
    const uint8_t *base = static_cast<const uint8_t *>(a->map);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | base[i];
    if (hlen > a->map_bytes - 8) throw std::runtime_error(path + ": header length beyond the file");
    JsonParser jp{reinterpret_cast<const char *>(base + 8), reinterpret_cast<const char *>(base + 8 + hlen),
                  "safetensors header"};
    const Json h = jp.value();
    if (h.kind != Json::Obj) throw std::runtime_error(path + ": safetensors header is not an object");
    a->data = base + 8 + hlen;
    const size_t data_bytes = a->map_bytes - 8 - hlen;
    for (const auto &kv : h.obj) {
        if (kv.first == "__metadata__") {
            for (const auto &m : kv.second.obj)
                if (m.second.kind == Json::Str) a->meta[m.first] = m.second.str;
            continue;
        }
        const Json &t = kv.second;
        auto field = [&](const char *k) -> const Json & {
            auto it = t.obj.find(k);
            if (it == t.obj.end()) throw std::runtime_error("tensor \"" + kv.first + "\": missing " + k);
            return it->second;
        };
        XdnaWeightArena::Tensor x;
        const std::string dt = field("dtype").str;
        if (dt == "F32") x.dtype = 0;
        else if (dt == "BF16") x.dtype = 1;
        else throw std::runtime_error("unexpected arena dtype " + dt + " (tensor \"" + kv.first + "\")");
        size_t n = 1;
        for (const Json &d : field("shape").arr) {
            x.shape.push_back((int64_t)as_u64(d, "shape"));
            n *= (size_t)x.shape.back();
        }
        const Json &off = field("data_offsets");
        if (off.arr.size() != 2) throw std::runtime_error("tensor \"" + kv.first + "\": bad data_offsets");
        x.begin = as_u64(off.arr[0], "data_offsets");
        x.end = as_u64(off.arr[1], "data_offsets");
        if (x.end < x.begin || x.end > data_bytes || x.end - x.begin != n * (x.dtype ? 2 : 4))
            throw std::runtime_error("tensor \"" + kv.first + "\": data_offsets disagree with shape or file size");
        a->tensors[kv.first] = x;
        a->names.push_back(kv.first);
    }
    const std::string arch = a->meta.count("arch") ? a->meta["arch"] : "";
    if (expect_arch && arch != expect_arch)
        throw std::runtime_error("arena arch \"" + arch + "\" != expected \"" + expect_arch + "\"");
    const std::string ver = a->meta.count("format_version") ? a->meta["format_version"] : "0";
    if (ver != "1") throw std::runtime_error("arena format_version " + ver + " != 1 (rebake)");
    return a.release();
}

bool is_directory(const std::string &p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

// name -> (shape, f32 data) from an arena or an npy directory
struct Store {
    XdnaWeightArena *arena = nullptr;
    std::string dir;
    void get(const std::string &name, std::vector<size_t> &shape, std::vector<float> &data) const {
        if (arena) {
            const auto &t = arena->get(name);
            shape.assign(t.shape.begin(), t.shape.end());
            data.resize(arena->count(t));
            arena->read_f32(t, data.data());
        } else {
            xdna::read_npy_f32(dir + "/" + name + ".npy", shape, data);
        }
    }
    bool has(const std::string &name) const {
        if (arena) return arena->tensors.count(name) != 0;
        std::ifstream f(dir + "/" + name + ".npy");
        return (bool)f;
    }
};

}  // namespace

extern "C" {

XdnaWeightArena *xdna_weights_open(const char *path, const char *expect_arch) {
    if (!path) {
        set_last_error_message("xdna_weights_open: path is null");
        return nullptr;
    }
    try {
        return open_arena(path, expect_arch);
    } catch (const std::exception &e) {
        set_last_error_message(std::string("xdna_weights_open: ") + e.what());
        return nullptr;
    }
}

void xdna_weights_close(XdnaWeightArena *a) { delete a; }

int xdna_weights_count(const XdnaWeightArena *a) { return a ? (int)a->names.size() : -1; }

const char *xdna_weights_name(const XdnaWeightArena *a, int i) {
    return a && i >= 0 && i < (int)a->names.size() ? a->names[i].c_str() : nullptr;
}

const char *xdna_weights_meta(const XdnaWeightArena *a, const char *key) {
    if (!a || !key) return nullptr;
    auto it = a->meta.find(key);
    return it == a->meta.end() ? nullptr : it->second.c_str();
}

int xdna_weights_info(const XdnaWeightArena *a, const char *name, int *dtype, int64_t *shape, int max_dims) {
    if (!a || !name) {
        set_last_error_message("xdna_weights_info: null arena or name");
        return -1;
    }
    auto it = a->tensors.find(name);
    if (it == a->tensors.end()) {
        set_last_error_message(std::string("xdna_weights_info: tensor \"") + name + "\" not in the arena");
        return -1;
    }
    if (dtype) *dtype = it->second.dtype;
    const int nd = (int)it->second.shape.size();
    for (int d = 0; d < nd && d < max_dims && shape; d++) shape[d] = it->second.shape[d];
    return nd;
}

int xdna_weights_read_f32(const XdnaWeightArena *a, const char *name, float *out, size_t n) {
    if (!a || !name || !out) {
        set_last_error_message("xdna_weights_read_f32: null pointer");
        return -1;
    }
    try {
        const auto &t = a->get(name);
        if (n != a->count(t)) throw std::runtime_error(std::string("tensor \"") + name + "\" holds " +
                                                       std::to_string(a->count(t)) + " values, not " + std::to_string(n));
        a->read_f32(t, out);
        return 0;
    } catch (const std::exception &e) {
        set_last_error_message(std::string("xdna_weights_read_f32: ") + e.what());
        return -1;
    }
}

int xdna_weights_read_bf16(const XdnaWeightArena *a, const char *name, uint16_t *out, size_t n) {
    if (!a || !name || !out) {
        set_last_error_message("xdna_weights_read_bf16: null pointer");
        return -1;
    }
    try {
        const auto &t = a->get(name);
        if (t.dtype != 1) return 1;   // an F32 tensor has no raw bf16 form (arena.rs:86-100)
        if (n != a->count(t)) throw std::runtime_error(std::string("tensor \"") + name + "\" holds " +
                                                       std::to_string(a->count(t)) + " values, not " + std::to_string(n));
        std::memcpy(out, a->data + t.begin, n * 2);
        return 0;
    } catch (const std::exception &e) {
        set_last_error_message(std::string("xdna_weights_read_bf16: ") + e.what());
        return -1;
    }
}

XdnaOptDecoder *xdna_opt_load(XdnaDevice *dev, const char *path, int max_ctx, int grid) {
    if (!dev || !path) {
        set_last_error_message("xdna_opt_load: null device or path");
        return nullptr;
    }
    std::unique_ptr<XdnaWeightArena> owned;
    try {
        Store s;
        if (is_directory(path)) s.dir = path;
        else {
            owned.reset(open_arena(path, "opt"));
            s.arena = owned.get();
        }
        std::vector<size_t> sh;
        std::vector<float> emb_tok, emb_pos, lnf_w, lnf_b, lm;
        auto want = [](const std::string &n, const std::vector<size_t> &shape, std::vector<size_t> expect) {
            if (shape != expect) {
                std::string a, b;
                for (size_t v : shape) a += std::to_string(v) + ",";
                for (size_t v : expect) b += std::to_string(v) + ",";
                throw std::runtime_error("tensor \"" + n + "\" has shape [" + a + "], expected [" + b + "]");
            }
        };
        s.get("embed_tokens", sh, emb_tok);
        if (sh.size() != 2) throw std::runtime_error("embed_tokens must be [vocab, d]");
        const size_t V = sh[0], D = sh[1];
        s.get("embed_positions", sh, emb_pos);
        if (sh.size() != 2 || sh[1] != D || sh[0] < 3) throw std::runtime_error("embed_positions must be [max_pos + 2, d]");
        const size_t P = sh[0];
        s.get("ln_final.weight", sh, lnf_w);
        want("ln_final.weight", sh, {D});
        s.get("ln_final.bias", sh, lnf_b);
        want("ln_final.bias", sh, {D});
        s.get("lm_head.weight", sh, lm);
        want("lm_head.weight", sh, {D, V});
        for (size_t v = 0; v < V; v++)
            for (size_t d = 0; d < D; d++)
                if (std::memcmp(&lm[d * V + v], &emb_tok[v * D + d], 4) != 0)
                    throw std::runtime_error("lm_head.weight is not embed_tokens transposed (an untied LM head is not "
                                             "supported)");
        lm.clear();
        lm.shrink_to_fit();
        int L = 0;
        while (s.has("L" + std::to_string(L) + "/q.weight")) L++;
        if (L == 0) throw std::runtime_error("no layers (L0/q.weight missing)");
        std::vector<std::vector<float>> keep;
        keep.reserve((size_t)L * 16);
        std::vector<XdnaOptLayer> layers(L);
        size_t F = 0;
        for (int l = 0; l < L; l++) {
            const std::string p = "L" + std::to_string(l) + "/";
            auto load = [&](const std::string &n, std::vector<size_t> expect) -> const float * {
                keep.emplace_back();
                s.get(p + n, sh, keep.back());
                want(p + n, sh, expect);
                return keep.back().data();
            };
            XdnaOptLayer &y = layers[l];
            y.wq = load("q.weight", {D, D});
            y.bq = load("q.bias", {D});
            y.wk = load("k.weight", {D, D});
            y.bk = load("k.bias", {D});
            y.wv = load("v.weight", {D, D});
            y.bv = load("v.bias", {D});
            y.wo = load("out.weight", {D, D});
            y.bo = load("out.bias", {D});
            y.ln1_w = load("ln_self.weight", {D});
            y.ln1_b = load("ln_self.bias", {D});
            y.ln2_w = load("ln_ffn.weight", {D});
            y.ln2_b = load("ln_ffn.bias", {D});
            if (l == 0) {
                std::vector<size_t> fs;
                std::vector<float> tmp;
                s.get(p + "fc1.weight", fs, tmp);
                if (fs.size() != 2 || fs[0] != D) throw std::runtime_error(p + "fc1.weight must be [d, ffn]");
                F = fs[1];
            }
            y.w1 = load("fc1.weight", {D, F});
            y.b1 = load("fc1.bias", {F});
            y.w2 = load("fc2.weight", {F, D});
            y.b2 = load("fc2.bias", {D});
        }
        XdnaOptConfig cfg;
        cfg.n_layers = L;
        cfg.d_model = (int)D;
        cfg.head_dim = 64;
        cfg.n_heads = (int)D / 64;
        cfg.ffn = (int)F;
        cfg.vocab = (int)V;
        cfg.max_pos = (int)P - 2;
        cfg.eps = 1e-5f;
        XdnaOptWeights w;
        w.emb_tok = emb_tok.data();
        w.emb_pos = emb_pos.data();
        w.lnf_w = lnf_w.data();
        w.lnf_b = lnf_b.data();
        w.layers = layers.data();
        if (max_ctx <= 0) max_ctx = std::min(cfg.max_pos, 2048);
        return xdna_opt_create(dev, &cfg, &w, max_ctx, grid);   // sets the error itself on failure
    } catch (const std::exception &e) {
        set_last_error_message(std::string("xdna_opt_load: ") + e.what());
        return nullptr;
    }
}

}  // extern "C"
