// runtime.cu -- the control plane behind npu_runtime_* (include/npu_engine.h), one worker per GPU.
//
// Replaces rust/npu-runtime (config.rs:6-45 desired state, registry.rs:26-78 load / unload /
// caps, reconcile.rs:11-31, select.rs:5-26 model resolution, actor.rs:23-96 the device actor,
// http.rs:55-66 the model list JSON) and its C surface rust/npu-capi/src/lib.rs:125-214.
//
// The reference drives ONE NPU from one actor thread.  Here every GPU gets its own worker thread
// with its own registry: a reconcile loads one replica of every configured model on every
// worker's GPU (in parallel across GPUs), and each request goes to the worker with the fewest
// requests in flight (ties broken round robin), where it runs on that GPU's replica.  A model's
// buffers and kernels are only ever touched by its worker thread, so requests on one GPU are
// serialised exactly like the reference's actor, and requests on different GPUs run at once.
//
// * Config (engine TOML): [server] port / memory_ceiling_mb / max_resident (all three when the
//   table is present, as ServerCfg in config.rs), [defaults] asr / embed, [[model]] name /
//   scenario.  A missing file is the empty default config.  One key beyond the reference's:
//   `[server] gpus = N` -- workers on CUDA devices 0..N-1 (default: every visible device, at
//   least one worker).  `port` is read and kept but nothing listens: HTTP is out of scope.
// * Caps per GPU: max_resident models and memory_ceiling_mb of device memory, a replica's size
//   being the device memory its load took (cudaMemGetInfo before and after, on its GPU).
// * Test loader: when the environment variable XDNA_RUNTIME_MOCK is set at npu_runtime_start,
//   models come from its table instead of scenarios (the reference's loader::mock::MockLoader,
//   loader.rs:32-60): "name=embed:BYTES;name=asr:BYTES;name=!MESSAGE" (a load that fails with
//   MESSAGE).  A mock embedder returns 8 floats, the first the GPU ordinal of the worker that
//   served the request; a mock recogniser returns "mock-text".  No CUDA call is made then.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <future>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/npu_engine.h"
#include "capi_internal.h"
#include "toml.h"

namespace {

using xdna::Toml;

constexpr int KIND_ASR = 0, KIND_EMBED = 1;
const char *kind_name(int k) { return k == KIND_ASR ? "asr" : "embed"; }

// an EngineError: the message is already its Display form ("load failed: ...", api.rs:20-31)
struct EngineError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// ------------------------------------------------------------------------------ config
struct ModelCfg {
    std::string name, scenario;
};
struct ServerCfg {
    long port = 11434, memory_ceiling_mb = 4096, max_resident = 1, gpus = 0;
};
struct Config {
    ServerCfg server;
    std::string def_asr, def_embed;   // empty: none
    std::vector<ModelCfg> models;
};

Config parse_config(const std::string &text) {
    Toml t;
    const std::string e = t.parse(text);
    if (!e.empty()) throw std::runtime_error(e);
    Config c;
    if (t.has_table("server")) {
        c.server.port = t.integer("server.port");
        c.server.memory_ceiling_mb = t.integer("server.memory_ceiling_mb");
        c.server.max_resident = t.integer("server.max_resident");
        if (t.has("server.gpus")) c.server.gpus = t.integer("server.gpus");
        if (c.server.port < 0 || c.server.port > 65535)
            throw std::runtime_error("invalid value for `server.port`: expected a u16");
        if (c.server.memory_ceiling_mb < 0 || c.server.max_resident < 0 || c.server.gpus < 0)
            throw std::runtime_error("invalid value: server sizes must not be negative");
    }
    if (t.has("defaults.asr")) c.def_asr = t.req_str("defaults.asr");
    if (t.has("defaults.embed")) c.def_embed = t.req_str("defaults.embed");
    for (int i = 0; i < t.count("model"); i++) {
        const std::string p = "model[" + std::to_string(i) + "].";
        c.models.push_back(ModelCfg{t.req_str(p + "name"), t.req_str(p + "scenario")});
    }
    return c;
}

// Config::load (config.rs:27-34): a missing file is the default (empty) config
Config load_config(const std::string &path) {
    FILE *fp = std::fopen(path.c_str(), "rb");
    if (!fp) {
        if (errno == ENOENT) return Config();
        throw std::runtime_error(path + ": " + std::strerror(errno));
    }
    std::string text;
    char buf[4096];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, fp)) > 0) text.append(buf, n);
    std::fclose(fp);
    try {
        return parse_config(text);
    } catch (const std::exception &e) {
        throw std::runtime_error(path + ": " + e.what());
    }
}

// ------------------------------------------------------------------------------ models
struct Inference {
    virtual ~Inference() = default;
    virtual int kind() const = 0;
    virtual uint64_t bo_bytes() const = 0;
    virtual std::string transcribe(const int16_t *pcm, size_t n, uint32_t sr) = 0;
    virtual std::vector<float> embed(const std::string &text) = 0;
};

struct EngineModel : Inference {
    NpuModel *m;
    uint64_t bytes;
    EngineModel(NpuModel *m_, uint64_t b) : m(m_), bytes(b) {}
    ~EngineModel() override { npu_model_free(m); }
    int kind() const override { return npu_model_kind(m); }
    uint64_t bo_bytes() const override { return bytes; }
    std::string transcribe(const int16_t *pcm, size_t n, uint32_t sr) override {
        char *r = npu_transcribe(m, pcm, n, sr);
        if (!r) throw EngineError(npu_last_error());
        std::string s(r);
        npu_string_free(r);
        return s;
    }
    std::vector<float> embed(const std::string &text) override {
        const int dim = npu_embed(m, text.c_str(), nullptr, 0);
        if (dim < 0) throw EngineError(npu_last_error());
        std::vector<float> v((size_t)dim);
        if (npu_embed(m, text.c_str(), v.data(), v.size()) < 0) throw EngineError(npu_last_error());
        return v;
    }
};

struct MockModel : Inference {
    int k, ordinal;
    uint64_t bytes;
    MockModel(int k_, uint64_t b, int o) : k(k_), ordinal(o), bytes(b) {}
    int kind() const override { return k; }
    uint64_t bo_bytes() const override { return bytes; }
    std::string transcribe(const int16_t *, size_t, uint32_t) override {
        if (k != KIND_ASR) throw EngineError("wrong model kind: wanted asr, got embed");
        return "mock-text";
    }
    std::vector<float> embed(const std::string &) override {
        if (k != KIND_EMBED) throw EngineError("wrong model kind: wanted embed, got asr");
        std::vector<float> v(8, 0.0f);
        v[0] = (float)ordinal;
        return v;
    }
};

struct Loader {
    virtual ~Loader() = default;
    virtual bool uses_device() const = 0;
    virtual std::unique_ptr<Inference> load(const ModelCfg &cfg, int ordinal) = 0;
};

// npu_engine::Model::load_in through npu_model_load_on, on the worker's GPU (current already)
struct EngineLoader : Loader {
    int n_devices;
    explicit EngineLoader(int n) : n_devices(n) {}
    bool uses_device() const override { return true; }
    std::unique_ptr<Inference> load(const ModelCfg &cfg, int ordinal) override {
        if (ordinal >= n_devices) throw EngineError("device error: no CUDA device " + std::to_string(ordinal));
        size_t free0 = 0, free1 = 0, total = 0;
        cudaMemGetInfo(&free0, &total);
        NpuModel *m = npu_model_load_on(cfg.scenario.c_str(), ordinal);
        if (!m) throw EngineError(npu_last_error());
        cudaMemGetInfo(&free1, &total);
        return std::unique_ptr<Inference>(new EngineModel(m, free0 > free1 ? (uint64_t)(free0 - free1) : 0));
    }
};

struct MockLoader : Loader {
    struct Item {
        bool ok;
        int kind;
        uint64_t bytes;
        std::string err;
    };
    std::map<std::string, Item> table;
    explicit MockLoader(const std::string &spec) {
        std::stringstream ss(spec);
        std::string e;
        while (std::getline(ss, e, ';')) {
            const size_t eq = e.find('=');
            if (eq == std::string::npos) continue;
            const std::string name = e.substr(0, eq), v = e.substr(eq + 1);
            Item it{true, KIND_EMBED, 0, ""};
            if (!v.empty() && v[0] == '!') {
                it.ok = false;
                it.err = v.substr(1);
            } else {
                const size_t c = v.find(':');
                it.kind = v.substr(0, c) == "asr" ? KIND_ASR : KIND_EMBED;
                it.bytes = c == std::string::npos ? 0 : std::strtoull(v.c_str() + c + 1, nullptr, 10);
            }
            table[name] = it;
        }
    }
    bool uses_device() const override { return false; }
    std::unique_ptr<Inference> load(const ModelCfg &cfg, int ordinal) override {
        auto it = table.find(cfg.name);
        if (it == table.end()) throw EngineError("load failed: no mock entry for " + cfg.name);
        if (!it->second.ok) throw EngineError("load failed: " + it->second.err);
        return std::unique_ptr<Inference>(new MockModel(it->second.kind, it->second.bytes, ordinal));
    }
};

// ------------------------------------------------------------------------------ registry
enum LoadState { LOADED, FAILED, UNLOADED };
struct Status {
    std::string name;
    LoadState state = UNLOADED;
    std::string detail;
    int kind = -1;   // -1: unknown
    uint64_t bo_bytes = 0;
};
struct Entry {
    ModelCfg cfg;
    std::unique_ptr<Inference> model;
    Status st;
};

// registry.rs:26-78, for one GPU
struct Registry {
    std::vector<Entry> entries;

    Inference *get_loaded(const std::string &name) const {
        for (const Entry &e : entries)
            if (e.cfg.name == name) return e.model.get();
        return nullptr;
    }
    uint64_t resident_bytes() const {
        uint64_t s = 0;
        for (const Entry &e : entries)
            if (e.model) s += e.model->bo_bytes();
        return s;
    }
    long resident_count() const {
        long n = 0;
        for (const Entry &e : entries) n += e.model != nullptr;
        return n;
    }
    void try_load(const ModelCfg &cfg, Loader &loader, const ServerCfg &srv, int ordinal) {
        if (resident_count() >= srv.max_resident) {
            set_failed(cfg, "over max_resident (" + std::to_string(srv.max_resident) + ")");
            return;
        }
        std::unique_ptr<Inference> m;
        try {
            m = loader.load(cfg, ordinal);
        } catch (const std::exception &e) {
            set_failed(cfg, e.what());
            return;
        }
        const uint64_t bo = m->bo_bytes();
        if (resident_bytes() + bo > (uint64_t)srv.memory_ceiling_mb * 1024 * 1024) {
            set_failed(cfg, "over memory_ceiling");
            return;
        }
        Entry e;
        e.cfg = cfg;
        e.st = Status{cfg.name, LOADED, "", m->kind(), bo};
        e.model = std::move(m);
        upsert(std::move(e));
    }
    void unload(const std::string &name) {
        entries.erase(std::remove_if(entries.begin(), entries.end(), [&](const Entry &e) { return e.cfg.name == name; }),
                      entries.end());
    }
    void set_failed(const ModelCfg &cfg, const std::string &detail) {
        Entry e;
        e.cfg = cfg;
        e.st = Status{cfg.name, FAILED, detail, -1, 0};
        upsert(std::move(e));
    }
    void upsert(Entry &&e) {
        for (Entry &x : entries)
            if (x.cfg.name == e.cfg.name) {
                x = std::move(e);
                return;
            }
        entries.push_back(std::move(e));
    }
};

// reconcile.rs:11-31: drop what the config no longer names, (re)load what is new, failed or
// changed, keep the rest
void reconcile(const Config &cfg, Registry &reg, Loader &loader, int ordinal) {
    std::vector<std::string> drop;
    for (const Entry &e : reg.entries) {
        bool want = false;
        for (const ModelCfg &m : cfg.models) want |= m.name == e.cfg.name;
        if (!want) drop.push_back(e.cfg.name);
    }
    for (const std::string &n : drop) reg.unload(n);
    for (const ModelCfg &m : cfg.models) {
        const Entry *ex = nullptr;
        for (const Entry &e : reg.entries)
            if (e.cfg.name == m.name) ex = &e;
        const bool needs = !ex || !ex->model || ex->cfg.scenario != m.scenario;
        if (!needs) continue;
        reg.unload(m.name);
        reg.try_load(m, loader, cfg.server, ordinal);
    }
}

// select.rs:5-26: an explicit name must be loaded with the right kind; else the configured
// default of the capability, else the one loaded model of that capability
std::string resolve(const Config &cfg, const Registry &reg, int cap, const char *want) {
    if (want) {
        const Inference *m = reg.get_loaded(want);
        if (!m) throw EngineError(std::string("load failed: model \"") + want + "\" not loaded");
        if (m->kind() != cap)
            throw EngineError(std::string("wrong model kind: wanted ") + kind_name(cap) + ", got " + kind_name(m->kind()));
        return want;
    }
    const std::string &dflt = cap == KIND_ASR ? cfg.def_asr : cfg.def_embed;
    if (!dflt.empty()) {
        const Inference *m = reg.get_loaded(dflt);
        if (m && m->kind() == cap) return dflt;
    }
    std::vector<std::string> of_cap;
    for (const Entry &e : reg.entries)
        if (e.model && e.model->kind() == cap) of_cap.push_back(e.cfg.name);
    if (of_cap.size() == 1) return of_cap[0];
    if (of_cap.empty()) throw EngineError(std::string("unsupported: no ") + kind_name(cap) + " model loaded");
    throw EngineError(std::string("unsupported: model required for ") + kind_name(cap) + " (multiple loaded)");
}

// ------------------------------------------------------------------------------ workers
// One GPU's actor (actor.rs:23-46): a thread with that GPU current, a FIFO of tasks and the
// registry only it touches.  Models are freed on the thread too, with their GPU current.
struct Worker {
    int ordinal;
    bool set_device;
    Registry reg;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<std::function<void()>> q;
    bool stopping = false;
    std::atomic<int> pending{0};
    std::thread th;

    Worker(int o, bool dev) : ordinal(o), set_device(dev) { th = std::thread([this] { run(); }); }
    void run() {
        if (set_device) cudaSetDevice(ordinal);
        for (;;) {
            std::function<void()> f;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stopping || !q.empty(); });
                if (q.empty()) break;   // stopping and drained
                f = std::move(q.front());
                q.pop_front();
            }
            f();
            pending--;
        }
        reg.entries.clear();
    }
    template <class F>
    auto submit(F f) -> std::future<decltype(f())> {
        auto task = std::make_shared<std::packaged_task<decltype(f())()>>(std::move(f));
        auto fut = task->get_future();
        pending++;
        {
            std::lock_guard<std::mutex> lk(mu);
            q.emplace_back([task] { (*task)(); });
        }
        cv.notify_one();
        return fut;
    }
    void stop() {
        {
            std::lock_guard<std::mutex> lk(mu);
            stopping = true;
        }
        cv.notify_one();
        if (th.joinable()) th.join();
    }
};

std::string json_escape(const std::string &s) {
    std::string o;
    for (unsigned char c : s) {
        switch (c) {
            case '"': o += "\\\""; break;
            case '\\': o += "\\\\"; break;
            case '\n': o += "\\n"; break;
            case '\r': o += "\\r"; break;
            case '\t': o += "\\t"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    std::snprintf(b, sizeof b, "\\u%04x", c);
                    o += b;
                } else {
                    o += (char)c;
                }
        }
    }
    return o;
}

char *dup_c(const std::string &s) {
    char *r = static_cast<char *>(std::malloc(s.size() + 1));
    if (r) std::memcpy(r, s.c_str(), s.size() + 1);
    return r;
}

}  // namespace

struct NpuRuntime {
    std::string cfg_path;
    std::mutex cfg_mu;
    std::shared_ptr<const Config> cfg;
    std::unique_ptr<Loader> loader;
    std::vector<std::unique_ptr<Worker>> workers;
    std::atomic<unsigned> rr{0};

    std::shared_ptr<const Config> config() {
        std::lock_guard<std::mutex> lk(cfg_mu);
        return cfg;
    }
    // the worker with the fewest requests in flight, scanning from a round-robin start
    Worker &pick() {
        const size_t n = workers.size(), s = rr++ % n;
        size_t best = s;
        for (size_t i = 1; i < n; i++) {
            const size_t k = (s + i) % n;
            if (workers[k]->pending.load() < workers[best]->pending.load()) best = k;
        }
        return *workers[best];
    }
    // reconcile every GPU's registry against `c` (the GPUs load in parallel)
    void reconcile_all(const std::shared_ptr<const Config> &c) {
        std::vector<std::future<void>> fs;
        for (auto &w : workers) {
            Worker *wp = w.get();
            Loader *ld = loader.get();
            fs.push_back(wp->submit([wp, ld, c] { reconcile(*c, wp->reg, *ld, wp->ordinal); }));
        }
        for (auto &f : fs) f.get();
    }
    ~NpuRuntime() {
        for (auto &w : workers) w->stop();
    }
};

extern "C" {

NpuRuntime *npu_runtime_start(const char *config_path) {
    try {
        if (!config_path) { npu_set_last_error("config_path is null"); return nullptr; }
        std::unique_ptr<NpuRuntime> rt(new NpuRuntime());
        rt->cfg_path = config_path;
        auto cfg = std::make_shared<const Config>(load_config(rt->cfg_path));
        rt->cfg = cfg;
        const char *mock = std::getenv("XDNA_RUNTIME_MOCK");
        int ndev = 0;
        if (mock) {
            rt->loader.reset(new MockLoader(mock));
        } else {
            if (cudaGetDeviceCount(&ndev) != cudaSuccess) {
                ndev = 0;
                cudaGetLastError();
            }
            rt->loader.reset(new EngineLoader(ndev));
        }
        const int n = cfg->server.gpus > 0 ? (int)cfg->server.gpus : std::max(1, ndev);
        for (int i = 0; i < n; i++)
            rt->workers.emplace_back(new Worker(i, rt->loader->uses_device() && i < ndev));
        rt->reconcile_all(cfg);
        return rt.release();
    } catch (const std::exception &e) {
        npu_set_last_error(e.what());
        return nullptr;
    } catch (...) {
        npu_set_last_error("panic in npu_runtime_start");
        return nullptr;
    }
}

char *npu_runtime_transcribe(NpuRuntime *rt, const char *model, const int16_t *pcm, uintptr_t n,
                             uint32_t sample_rate) {
    try {
        if (!rt) { npu_set_last_error("runtime is null"); return nullptr; }
        if (!pcm && n != 0) { npu_set_last_error("pcm is null"); return nullptr; }
        auto cfg = rt->config();
        Worker &w = rt->pick();
        Worker *wp = &w;
        std::string want;
        const bool has = model != nullptr;
        if (has) want = model;
        std::vector<int16_t> samples(pcm, pcm + (pcm ? n : 0));
        auto fut = w.submit([wp, cfg, has, want, samples = std::move(samples), sample_rate]() -> std::string {
            const std::string name = resolve(*cfg, wp->reg, KIND_ASR, has ? want.c_str() : nullptr);
            return wp->reg.get_loaded(name)->transcribe(samples.data(), samples.size(), sample_rate);
        });
        const std::string text = fut.get();
        char *r = dup_c(text);
        if (!r) npu_set_last_error("out of host memory");
        return r;
    } catch (const std::exception &e) {
        npu_set_last_error(e.what());
        return nullptr;
    } catch (...) {
        npu_set_last_error("panic in npu_runtime_transcribe");
        return nullptr;
    }
}

int npu_runtime_embed(NpuRuntime *rt, const char *model, const char *text, float *out, uintptr_t out_cap) {
    try {
        if (!rt) { npu_set_last_error("runtime is null"); return -1; }
        if (!text) { npu_set_last_error("text is null"); return -1; }
        auto cfg = rt->config();
        Worker &w = rt->pick();
        Worker *wp = &w;
        const bool has = model != nullptr;
        const std::string want = has ? model : "", t = text;
        auto fut = w.submit([wp, cfg, has, want, t]() -> std::vector<float> {
            const std::string name = resolve(*cfg, wp->reg, KIND_EMBED, has ? want.c_str() : nullptr);
            return wp->reg.get_loaded(name)->embed(t);
        });
        const std::vector<float> v = fut.get();
        if (out && out_cap > 0) std::memcpy(out, v.data(), sizeof(float) * std::min<size_t>(v.size(), out_cap));
        return (int)v.size();
    } catch (const std::exception &e) {
        npu_set_last_error(e.what());
        return -1;
    } catch (...) {
        npu_set_last_error("panic in npu_runtime_embed");
        return -1;
    }
}

int npu_runtime_reload(NpuRuntime *rt) {
    try {
        if (!rt) { npu_set_last_error("runtime is null"); return -1; }
        auto cfg = std::make_shared<const Config>(load_config(rt->cfg_path));
        {
            std::lock_guard<std::mutex> lk(rt->cfg_mu);
            rt->cfg = cfg;
        }
        rt->reconcile_all(cfg);
        return 0;
    } catch (const std::exception &e) {
        npu_set_last_error(e.what());
        return -1;
    } catch (...) {
        npu_set_last_error("panic in npu_runtime_reload");
        return -1;
    }
}

// http.rs:55-66, one object per model: its state over the GPUs (loaded if any replica is),
// plus "replicas" (GPUs holding it) and "devices" (their ordinals); bo_bytes sums the replicas
char *npu_runtime_models_json(NpuRuntime *rt) {
    try {
        if (!rt) { npu_set_last_error("runtime is null"); return nullptr; }
        std::vector<std::future<std::vector<Status>>> fs;
        for (auto &w : rt->workers) {
            Worker *wp = w.get();
            fs.push_back(wp->submit([wp] {
                std::vector<Status> s;
                for (const Entry &e : wp->reg.entries) s.push_back(e.st);
                return s;
            }));
        }
        std::vector<std::string> order;
        std::map<std::string, std::vector<std::pair<int, Status>>> by;
        for (size_t i = 0; i < fs.size(); i++)
            for (Status &s : fs[i].get()) {
                if (!by.count(s.name)) order.push_back(s.name);
                by[s.name].push_back({(int)i, s});
            }
        std::string data;
        for (const std::string &name : order) {
            int replicas = 0, kind = -1;
            uint64_t bo = 0;
            std::string devices, detail;
            bool any_failed = false;
            for (auto &p : by[name]) {
                const Status &s = p.second;
                if (s.state == LOADED) {
                    devices += (replicas ? "," : "") + std::to_string(p.first);
                    replicas++;
                    bo += s.bo_bytes;
                    if (kind < 0) kind = s.kind;
                } else if (s.state == FAILED && !any_failed) {
                    any_failed = true;
                    detail = s.detail;
                }
            }
            const char *state = replicas ? "loaded" : any_failed ? "failed" : "unloaded";
            if (replicas) detail.clear();
            if (!data.empty()) data += ',';
            data += "{\"id\":\"" + json_escape(name) + "\",\"object\":\"model\",\"kind\":\"" +
                    (kind < 0 ? "unknown" : kind_name(kind)) + "\",\"state\":\"" + state + "\",\"detail\":\"" +
                    json_escape(detail) + "\",\"bo_bytes\":" + std::to_string(bo) +
                    ",\"replicas\":" + std::to_string(replicas) + ",\"devices\":[" + devices + "]}";
        }
        char *r = dup_c("{\"object\":\"list\",\"data\":[" + data + "]}");
        if (!r) npu_set_last_error("out of host memory");
        return r;
    } catch (const std::exception &e) {
        npu_set_last_error(e.what());
        return nullptr;
    } catch (...) {
        npu_set_last_error("panic in npu_runtime_models_json");
        return nullptr;
    }
}

void npu_runtime_stop(NpuRuntime *rt) {
    try {
        delete rt;
    } catch (...) {
    }
}

}  // extern "C"
