// adapter.cpp -- LoRA merge at load (src/adapter-merge.h): an adapter's low-rank deltas folded into
// the staged GGUF weights before the loader builds its resident copies, so inference runs on the
// merged model at no extra cost.
//
// Input formats (adapter_merge, adapter-merge.h:960-1011): a PEFT directory
// (adapter_model.safetensors + adapter_config.json with lora_alpha) or one safetensors file
// (ComfyUI). Keys: base_model.model.<path>.lora_A/B[.default].weight, <path>.lora_down/up.weight,
// diffusion_model.<path>...; per-tensor alpha scalars <path>.alpha (lora_base_name / lora_is_a /
// lora_is_b, :88-130). Scaling = alpha / rank * scale, alpha from the tensor, else the config,
// else the rank (:586-597). A LyCORIS LoKr payload (*.lokr_w1 / *.lokr_w2*) goes to the LoKr
// merge (Kronecker delta, optional DoRA, lokr_merge below).
//
// Per merged tensor, on the device: dequantise the staged base (acb_get_rows, bit-exact), add the
// bf16-rounded delta (acb_lora_delta_add / acb_lokr_delta_add), requantise into the staged bytes
// (acb_requant). A and B
// are read as f32 from F32 / BF16 / F16 and rounded to bf16 on the host, as PEFT does.
#include "adapter.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "host_common.h"

namespace acb {
namespace {

struct StEntry {
    std::string          name, dtype;
    std::vector<int64_t> shape;
    size_t               begin = 0, end = 0;  // within the data section
};

// A safetensors file: 8-byte little-endian header length, a JSON object of
// name -> {"dtype", "shape", "data_offsets"} (and "__metadata__"), then the data.
struct StFile {
    int                  fd   = -1;
    uint8_t *            map  = nullptr;
    size_t               size = 0, data_off = 0;
    std::vector<StEntry> entries;
    std::map<std::string, std::string> meta;  // __metadata__ (string values)
    std::string          err;

    ~StFile() {
        if (map) {
            munmap(map, size);
        }
        if (fd >= 0) {
            close(fd);
        }
    }

    const uint8_t * data(const StEntry & e) const { return map + data_off + e.begin; }
    bool            open_file(const std::string & path);
};

// A small JSON reader for the safetensors header (objects, arrays, strings, numbers).
struct Json {
    const char * p;
    const char * e;
    bool         ok = true;

    void ws() {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) {
            p++;
        }
    }
    bool eat(char c) {
        ws();
        if (p < e && *p == c) {
            p++;
            return true;
        }
        return false;
    }
    std::string str() {
        ws();
        std::string s;
        if (p >= e || *p != '"') {
            ok = false;
            return s;
        }
        p++;
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) {
                p++;
            }
            s.push_back(*p++);
        }
        if (p < e) {
            p++;
        } else {
            ok = false;
        }
        return s;
    }
    int64_t num() {
        ws();
        char *        q = nullptr;
        const int64_t v = strtoll(p, &q, 10);
        if (q == p) {
            ok = false;
        }
        p = q;
        while (p < e && (*p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+' || (*p >= '0' && *p <= '9'))) {
            p++;
        }
        return v;
    }
    void skip() {  // any value
        ws();
        if (p >= e) {
            ok = false;
            return;
        }
        if (*p == '"') {
            str();
        } else if (*p == '{' || *p == '[') {
            const char open = *p, close = open == '{' ? '}' : ']';
            p++;
            if (eat(close)) {
                return;
            }
            do {
                if (open == '{') {
                    str();
                    if (!eat(':')) {
                        ok = false;
                        return;
                    }
                }
                skip();
            } while (ok && eat(','));
            if (!eat(close)) {
                ok = false;
            }
        } else {
            while (p < e && *p != ',' && *p != '}' && *p != ']') {
                p++;
            }
        }
    }
};

bool StFile::open_file(const std::string & path) {
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return false;
    }
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        err = "not a safetensors file: " + path;
        return false;
    }
    size = (size_t) sb.st_size;
    map  = (uint8_t *) mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        map = nullptr;
        err = "cannot map " + path;
        return false;
    }
    uint64_t hl = 0;
    memcpy(&hl, map, 8);
    if (hl > size - 8) {
        err = "truncated safetensors header";
        return false;
    }
    data_off = 8 + (size_t) hl;
    Json j{ (const char *) map + 8, (const char *) map + 8 + hl };
    if (!j.eat('{')) {
        err = "malformed safetensors header";
        return false;
    }
    if (!j.eat('}')) {
        do {
            StEntry t;
            t.name = j.str();
            if (!j.eat(':')) {
                j.ok = false;
                break;
            }
            if (t.name == "__metadata__") {
                if (!j.eat('{')) {
                    j.ok = false;
                    break;
                }
                if (!j.eat('}')) {
                    do {
                        const std::string k = j.str();
                        if (!j.eat(':')) {
                            j.ok = false;
                            break;
                        }
                        j.ws();
                        if (j.p < j.e && *j.p == '"') {
                            meta[k] = j.str();
                        } else {
                            j.skip();
                        }
                    } while (j.ok && j.eat(','));
                    if (j.ok && !j.eat('}')) {
                        j.ok = false;
                    }
                }
                continue;
            }
            if (!j.eat('{')) {
                j.ok = false;
                break;
            }
            do {
                const std::string k = j.str();
                if (!j.eat(':')) {
                    j.ok = false;
                    break;
                }
                if (k == "dtype") {
                    t.dtype = j.str();
                } else if (k == "shape") {
                    if (!j.eat('[')) {
                        j.ok = false;
                        break;
                    }
                    if (!j.eat(']')) {
                        do {
                            t.shape.push_back(j.num());
                        } while (j.ok && j.eat(','));
                        if (!j.eat(']')) {
                            j.ok = false;
                        }
                    }
                } else if (k == "data_offsets") {
                    if (!j.eat('[')) {
                        j.ok = false;
                        break;
                    }
                    t.begin = (size_t) j.num();
                    j.eat(',');
                    t.end = (size_t) j.num();
                    if (!j.eat(']')) {
                        j.ok = false;
                    }
                } else {
                    j.skip();
                }
            } while (j.ok && j.eat(','));
            if (!j.ok || !j.eat('}')) {
                j.ok = false;
                break;
            }
            if (t.end < t.begin || data_off + t.end > size) {
                err = "tensor '" + t.name + "' outside the file";
                return false;
            }
            entries.push_back(std::move(t));
        } while (j.ok && j.eat(','));
        if (j.ok && !j.eat('}')) {
            j.ok = false;
        }
    }
    if (!j.ok) {
        err = "malformed safetensors header";
        return false;
    }
    return true;
}

// lora_base_name (adapter-merge.h:88-120): the GGUF weight a LoRA key belongs to
std::string lora_base(const std::string & key) {
    std::string s = key;
    for (const char * pfx : { "base_model.model.", "diffusion_model." }) {
        const size_t n = strlen(pfx);
        if (s.compare(0, n, pfx) == 0) {
            s = s.substr(n);
            break;
        }
    }
    const size_t pos = s.find(".lora_");
    if (pos == std::string::npos) {
        return "";
    }
    s = s.substr(0, pos);
    if (s.compare(0, 8, "decoder.") != 0) {
        s = "decoder." + s;
    }
    return s + ".weight";
}

bool lora_a(const std::string & k) {
    return k.find(".lora_A.") != std::string::npos || k.find(".lora_down.") != std::string::npos;
}

bool lora_b(const std::string & k) {
    return k.find(".lora_B.") != std::string::npos || k.find(".lora_up.") != std::string::npos;
}

// "lora_alpha": <int> (else "alpha": <int>) of adapter_config.json (adapter_read_alpha, :132-185)
int config_alpha(const std::string & dir) {
    FILE * f = fopen((dir + "/adapter_config.json").c_str(), "rb");
    if (!f) {
        return 0;
    }
    std::string txt;
    char        buf[4096];
    size_t      n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) {
        txt.append(buf, n);
    }
    fclose(f);
    for (const char * key : { "\"lora_alpha\"", "\"alpha\"" }) {
        const size_t p = txt.find(key);
        if (p != std::string::npos) {
            const size_t c = txt.find(':', p + strlen(key));
            if (c != std::string::npos) {
                const int a = atoi(txt.c_str() + c + 1);
                if (a > 0) {
                    return a;
                }
            }
        }
    }
    return 0;
}

// F32 / BF16 / F16 safetensors data to f32 (adapter_to_f32, adapter-merge.h:59-86)
bool to_f32(const uint8_t * src, const std::string & dtype, size_t n, std::vector<float> & out) {
    out.resize(n);
    for (size_t i = 0; i < n; i++) {
        float v;
        if (dtype == "F32") {
            memcpy(&v, src + 4 * i, 4);
        } else if (dtype == "BF16") {
            uint16_t h;
            memcpy(&h, src + 2 * i, 2);
            v = host_bf16_to_f32(h);
        } else if (dtype == "F16") {
            uint16_t h;
            memcpy(&h, src + 2 * i, 2);
            v = host_f16_to_f32(h);
        } else {
            return false;
        }
        out[i] = v;
    }
    return true;
}

// the same, rounded to bf16 (PEFT's cast of A and B)
bool to_bf16_f32(const uint8_t * src, const std::string & dtype, size_t n, std::vector<float> & out) {
    if (!to_f32(src, dtype, n, out)) {
        return false;
    }
    for (float & v : out) {
        v = host_bf16_to_f32(host_f32_to_bf16(v));
    }
    return true;
}

int64_t numel(const StEntry & e) {
    int64_t n = 1;
    for (int64_t d : e.shape) {
        n *= d;
    }
    return n;
}

// __metadata__.lokr_config.linear_dim (adapter_read_lokr_dim, adapter-merge.h:187-218): the rank of
// monolithic LoKr modules; 0 when absent
int lokr_linear_dim(const StFile & f) {
    const auto it = f.meta.find("lokr_config");
    if (it == f.meta.end()) {
        return 0;
    }
    Json j{ it->second.data(), it->second.data() + it->second.size() };
    if (!j.eat('{') || j.eat('}')) {
        return 0;
    }
    do {
        const std::string k = j.str();
        if (!j.eat(':')) {
            return 0;
        }
        if (k == "linear_dim") {
            const int64_t v = j.num();
            return j.ok && v > 0 && v < (1 << 30) ? (int) v : 0;
        }
        j.skip();
    } while (j.ok && j.eat(','));
    return 0;
}

// LyCORIS LoKr merge (adapter_merge_lokr, adapter-merge.h:674-958): modules lycoris_<path> with
// lokr_w1 and either lokr_w2_a + lokr_w2_b (factorised, rank = w2_a's columns) or lokr_w2
// (monolithic, rank = lokr_config.linear_dim), alpha, optional dora_scale; target decoder.<path
// with dots>.weight (lokr_build_reverse_map, :278-306). Incomplete, ambiguous or misshapen modules
// are skipped, as the reference does with a warning.
acb_status lokr_merge(const StFile & f, float scale, WeightArena & staged, cudaStream_t st, int * n_merged) {
    struct Mod {
        const StEntry * w1 = nullptr;
        const StEntry * w2 = nullptr;
        const StEntry * w2a = nullptr;
        const StEntry * w2b = nullptr;
        const StEntry * alpha = nullptr;
        const StEntry * ds = nullptr;
    };
    std::map<std::string, Mod> mods;
    for (const StEntry & e : f.entries) {
        const size_t dot = e.name.rfind('.');
        if (dot == std::string::npos || e.name.compare(0, 8, "lycoris_") != 0) {
            continue;
        }
        const std::string pfx = e.name.substr(0, dot), sfx = e.name.substr(dot + 1);
        Mod &             m   = mods[pfx];
        if (sfx == "lokr_w1") {
            m.w1 = &e;
        } else if (sfx == "lokr_w2") {
            m.w2 = &e;
        } else if (sfx == "lokr_w2_a") {
            m.w2a = &e;
        } else if (sfx == "lokr_w2_b") {
            m.w2b = &e;
        } else if (sfx == "alpha") {
            m.alpha = &e;
        } else if (sfx == "dora_scale") {
            m.ds = &e;
        }
    }
    std::map<std::string, std::string> target;  // lycoris_<path with underscores> -> GGUF name
    for (const std::string & n : staged.names()) {
        const std::string sfx = ".weight";
        if (n.size() <= 8 + sfx.size() || n.compare(0, 8, "decoder.") != 0 ||
            n.compare(n.size() - sfx.size(), sfx.size(), sfx) != 0) {
            continue;
        }
        std::string path = n.substr(8, n.size() - 8 - sfx.size());
        for (char & ch : path) {
            ch = ch == '.' ? '_' : ch;
        }
        target["lycoris_" + path] = n;
    }
    const int          lokr_dim = lokr_linear_dim(f);
    DevBuf             d1, d2, dds, tmp, ids;
    std::vector<float> h1, h2, h2a, h2b, hds, hal;
    for (const auto & kv : mods) {
        const Mod & m      = kv.second;
        const bool  factor = m.w2a && m.w2b, mono = m.w2 != nullptr;
        const auto  tg     = target.find(kv.first);
        if (!m.w1 || !m.alpha || factor == mono || tg == target.end() || m.w1->shape.size() != 2) {
            continue;
        }
        DevTensor * t = staged.get(tg->second);
        if (!t) {
            continue;
        }
        const int64_t a = m.w1->shape[0], b = m.w1->shape[1];
        int64_t       c, d, r;
        if (factor) {
            if (m.w2a->shape.size() != 2 || m.w2b->shape.size() != 2 || m.w2a->shape[1] != m.w2b->shape[0]) {
                continue;
            }
            c = m.w2a->shape[0], r = m.w2a->shape[1], d = m.w2b->shape[1];
        } else {
            if (m.w2->shape.size() != 2 || lokr_dim <= 0) {
                continue;
            }
            c = m.w2->shape[0], d = m.w2->shape[1], r = lokr_dim;
        }
        if (a * c != t->N || b * d != t->K || numel(*m.alpha) != 1 ||
            !to_f32(f.data(*m.alpha), m.alpha->dtype, 1, hal) ||
            !to_f32(f.data(*m.w1), m.w1->dtype, (size_t) (a * b), h1)) {
            continue;
        }
        if (factor) {
            if (!to_f32(f.data(*m.w2a), m.w2a->dtype, (size_t) (c * r), h2a) ||
                !to_f32(f.data(*m.w2b), m.w2b->dtype, (size_t) (r * d), h2b)) {
                continue;
            }
            // W2 = w2_a . w2_b: exact products summed in double in ascending rank, rounded once
            std::vector<double> acc((size_t) (c * d), 0.0);
            for (int64_t q = 0; q < r; q++) {
                for (int64_t i = 0; i < c; i++) {
                    const double x = h2a[(size_t) (i * r + q)];
                    double *     o = &acc[(size_t) (i * d)];
                    const float * y = &h2b[(size_t) (q * d)];
                    for (int64_t l = 0; l < d; l++) {
                        o[l] += x * (double) y[l];
                    }
                }
            }
            h2.resize(acc.size());
            for (size_t i = 0; i < acc.size(); i++) {
                h2[i] = (float) acc[i];
            }
        } else if (!to_f32(f.data(*m.w2), m.w2->dtype, (size_t) (c * d), h2)) {
            continue;
        }
        const float * ds_dev = nullptr;
        if (m.ds) {
            if (m.ds->shape.empty() || m.ds->shape[0] != t->N || numel(*m.ds) != t->N ||
                !to_f32(f.data(*m.ds), m.ds->dtype, (size_t) t->N, hds)) {
                continue;
            }
            if (dds.bytes < hds.size() * 4) {
                ACB_TRY(dds.alloc(hds.size() * 4, false));
            }
            if (cudaMemcpyAsync(dds.p, hds.data(), hds.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
                return ACB_ERR_CUDA;
            }
            ds_dev = dds.as<float>();
        }
        const float scaling = hal[0] / (float) r;  // alpha / rank, on the small factor
        for (float & v : h1) {
            v = v * scaling;
        }
        const int64_t N = t->N, K = t->K;
        if (d1.bytes < h1.size() * 4) {
            ACB_TRY(d1.alloc(h1.size() * 4, false));
        }
        if (d2.bytes < h2.size() * 4) {
            ACB_TRY(d2.alloc(h2.size() * 4, false));
        }
        if (tmp.bytes < (size_t) (N * K) * 4) {
            ACB_TRY(tmp.alloc((size_t) (N * K) * 4, false));
        }
        if (ids.bytes < (size_t) N * 4) {
            ACB_TRY(ids.alloc((size_t) N * 4, false));
            std::vector<int32_t> iv((size_t) N);
            for (int64_t q = 0; q < N; q++) {
                iv[(size_t) q] = (int32_t) q;
            }
            cudaMemcpy(ids.p, iv.data(), iv.size() * 4, cudaMemcpyHostToDevice);
        }
        if (cudaMemcpyAsync(d1.p, h1.data(), h1.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d2.p, h2.data(), h2.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        const acb_stream_t as = (acb_stream_t) st;
        ACB_TRY(acb_get_rows(t->data, t->type, N, K, ids.as<int32_t>(), N, tmp.p, ACB_TYPE_F32, K, nullptr, as));
        ACB_TRY(acb_lokr_delta_add(tmp.as<float>(), N, K, d1.as<float>(), (int) a, (int) b, d2.as<float>(), (int) c,
                                   (int) d, scale, ds_dev, as));
        ACB_TRY(acb_requant(tmp.as<float>(), N, K, t->type, t->data, as));
        if (cudaStreamSynchronize(st) != cudaSuccess) {  // host buffers are reused by the next module
            return ACB_ERR_CUDA;
        }
        (*n_merged)++;
    }
    if (*n_merged == 0) {
        set_last_error("adapter: no LoKr module matched a weight of the model");
        return ACB_ERR_FORMAT;
    }
    return ACB_OK;
}

}  // namespace

acb_status adapter_merge(const char * adapter_path, float scale, WeightArena & staged, cudaStream_t st,
                         int * n_merged) {
    *n_merged = 0;
    struct stat sb;
    if (!adapter_path || stat(adapter_path, &sb) != 0) {
        set_last_error(std::string("adapter path does not exist: ") + (adapter_path ? adapter_path : "(null)"));
        return ACB_ERR_IO;
    }
    std::string sf, dir;
    if (S_ISDIR(sb.st_mode)) {
        dir = adapter_path;
        sf  = dir + "/adapter_model.safetensors";
    } else {
        sf              = adapter_path;
        const size_t s2 = sf.find_last_of('/');
        dir             = s2 == std::string::npos ? "." : sf.substr(0, s2);
    }
    StFile f;
    if (!f.open_file(sf)) {
        set_last_error("adapter: " + f.err);
        return ACB_ERR_IO;
    }
    for (const StEntry & e : f.entries) {  // adapter_detect_lokr (:321-330): one marker is enough
        if (e.name.find(".lokr_w1") != std::string::npos || e.name.find(".lokr_w2") != std::string::npos) {
            return lokr_merge(f, scale, staged, st, n_merged);
        }
    }
    const int                              alpha_cfg = config_alpha(dir);
    std::map<std::string, const StEntry *> amap, bmap;
    std::map<std::string, float>           alpha_of;
    for (const StEntry & e : f.entries) {
        const std::string sfx = ".alpha";
        if (e.name.size() > sfx.size() && e.name.compare(e.name.size() - sfx.size(), sfx.size(), sfx) == 0 &&
            e.dtype == "F32" && e.shape.empty() && e.end - e.begin == 4) {
            const std::string base = lora_base(e.name.substr(0, e.name.size() - sfx.size()) + ".lora_.x");
            if (!base.empty()) {
                float v;
                memcpy(&v, f.data(e), 4);
                alpha_of[base] = v;
            }
            continue;
        }
        const std::string base = lora_base(e.name);
        if (base.empty()) {
            continue;
        }
        if (lora_a(e.name)) {
            amap[base] = &e;
        } else if (lora_b(e.name)) {
            bmap[base] = &e;
        }
    }
    DevBuf             dA, dB, tmp, ids;
    std::vector<float> ha, hb;
    for (const auto & kv : amap) {
        const std::string & name = kv.first;
        const StEntry *     ea   = kv.second;
        const auto          ib   = bmap.find(name);
        DevTensor *         t    = staged.get(name);
        if (ib == bmap.end() || !t || ea->shape.size() != 2 || ib->second->shape.size() != 2) {
            continue;  // the reference skips such pairs with a warning
        }
        const StEntry * eb   = ib->second;
        const int64_t   rank = ea->shape[0], K = ea->shape[1], N = eb->shape[0];
        if (eb->shape[1] != rank || K != t->K || N != t->N) {
            continue;
        }
        float alpha = (float) rank;
        if (alpha_of.count(name)) {
            alpha = alpha_of[name];
        } else if (alpha_cfg > 0) {
            alpha = (float) alpha_cfg;
        }
        const float scaling = (alpha / (float) rank) * scale;
        if (!to_bf16_f32(f.data(*ea), ea->dtype, (size_t) (rank * K), ha) ||
            !to_bf16_f32(f.data(*eb), eb->dtype, (size_t) (N * rank), hb)) {
            continue;
        }
        if (dA.bytes < ha.size() * 4) {
            ACB_TRY(dA.alloc(ha.size() * 4, false));
        }
        if (dB.bytes < hb.size() * 4) {
            ACB_TRY(dB.alloc(hb.size() * 4, false));
        }
        if (tmp.bytes < (size_t) (N * K) * 4) {
            ACB_TRY(tmp.alloc((size_t) (N * K) * 4, false));
        }
        if (ids.bytes < (size_t) N * 4) {
            ACB_TRY(ids.alloc((size_t) N * 4, false));
            std::vector<int32_t> iv((size_t) N);
            for (int64_t r = 0; r < N; r++) {
                iv[(size_t) r] = (int32_t) r;
            }
            cudaMemcpy(ids.p, iv.data(), iv.size() * 4, cudaMemcpyHostToDevice);
        }
        if (cudaMemcpyAsync(dA.p, ha.data(), ha.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(dB.p, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        const acb_stream_t as = (acb_stream_t) st;
        ACB_TRY(acb_get_rows(t->data, t->type, N, K, ids.as<int32_t>(), N, tmp.p, ACB_TYPE_F32, K, nullptr, as));
        ACB_TRY(acb_lora_delta_add(tmp.as<float>(), N, K, dA.as<float>(), dB.as<float>(), (int) rank, scaling, as));
        ACB_TRY(acb_requant(tmp.as<float>(), N, K, t->type, t->data, as));
        if (cudaStreamSynchronize(st) != cudaSuccess) {  // host buffers are reused by the next pair
            return ACB_ERR_CUDA;
        }
        (*n_merged)++;
    }
    if (*n_merged == 0) {
        set_last_error("adapter: no LoRA pair matched a weight of the model");
        return ACB_ERR_FORMAT;
    }
    return ACB_OK;
}

}  // namespace acb
