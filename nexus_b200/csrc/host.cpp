// host.cpp -- host-side pieces of the backend: GGUF reader, host quantizers
// and the seeded synthetic-model writer (the role nexus-convert plays in the
// reference, tools/nexus-convert/main.rs).  Compiled with -ffp-contract=off so
// the shared quantizer arithmetic (quant_math.cuh) rounds like the reference.
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/nexus_cuda.h"
#include "gguf.h"
#include "quant_math.cuh"

namespace nx {

// ---------------------------------------------------------------------------
// GGUF reader
// ---------------------------------------------------------------------------
GgufFile::~GgufFile() {
    if (map_ && len_) munmap((void *)map_, len_);
}

namespace {
struct Cursor {
    const uint8_t *d;
    size_t len, pos;
    bool u32(uint32_t *v) {
        if (pos + 4 > len) return false;
        memcpy(v, d + pos, 4);
        pos += 4;
        return true;
    }
    bool u64(uint64_t *v) {
        if (pos + 8 > len) return false;
        memcpy(v, d + pos, 8);
        pos += 8;
        return true;
    }
    bool str(std::string *s) {
        uint64_t n;
        if (!u64(&n) || n > len - pos) return false;
        s->assign((const char *)d + pos, (size_t)n);
        pos += (size_t)n;
        return true;
    }
};
enum { VT_U8 = 0, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR, VT_U64, VT_I64, VT_F64 };
}  // namespace

int GgufFile::open(const std::string &path, std::string &err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return NEXUS_E_IO;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        err = "cannot stat " + path;
        return NEXUS_E_IO;
    }
    len_ = (size_t)st.st_size;
    if (len_) {
        void *p = mmap(nullptr, len_, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            ::close(fd);
            len_ = 0;
            err = "cannot mmap " + path;
            return NEXUS_E_IO;
        }
        map_ = (const uint8_t *)p;
    }
    ::close(fd);
    Cursor c{map_, len_, 0};
    if (len_ < 8 || memcmp(map_, "GGUF", 4) != 0) {
        err = "Invalid GGUF magic";
        return NEXUS_E_INVALID;
    }
    c.pos = 4;
    uint64_t tc, kc;
    if (!c.u32(&version_) || (version_ != 2 && version_ != 3)) {
        err = "Unsupported GGUF version";
        return NEXUS_E_INVALID;
    }
    if (!c.u64(&tc) || !c.u64(&kc)) {
        err = "Unexpected EOF reading counts";
        return NEXUS_E_TRUNCATED;
    }
    for (uint64_t k = 0; k < kc; k++) {
        std::string key;
        uint32_t vt;
        GgufValue v;
        if (!c.str(&key) || !c.u32(&vt)) {
            err = "Unexpected EOF reading metadata";
            return NEXUS_E_TRUNCATED;
        }
        if (vt > VT_F64) {
            err = "Unknown value type";
            return NEXUS_E_INVALID;
        }
        v.vtype = (int)vt;
        bool ok = true;
        switch (vt) {
        case VT_U8: case VT_I8: case VT_BOOL:
            if (c.pos + 1 > len_) { ok = false; break; }
            v.u = map_[c.pos];
            v.i = vt == VT_I8 ? (int8_t)map_[c.pos] : (int64_t)map_[c.pos];
            c.pos += 1;
            break;
        case VT_U16: case VT_I16: {
            if (c.pos + 2 > len_) { ok = false; break; }
            uint16_t x;
            memcpy(&x, map_ + c.pos, 2);
            v.u = x;
            v.i = vt == VT_I16 ? (int16_t)x : x;
            c.pos += 2;
            break;
        }
        case VT_U32: case VT_I32: case VT_F32: {
            uint32_t x;
            ok = c.u32(&x);
            v.u = x;
            v.i = (int32_t)x;
            v.f = u2f(x);
            break;
        }
        case VT_U64: case VT_I64: case VT_F64: {
            uint64_t x;
            ok = c.u64(&x);
            v.u = x;
            v.i = (int64_t)x;
            double f;
            memcpy(&f, &x, 8);
            v.f = f;
            break;
        }
        case VT_STR: ok = c.str(&v.s); break;
        case VT_ARR: {
            uint32_t at;
            uint64_t n;
            ok = c.u32(&at) && c.u64(&n) && at <= VT_F64;
            if (!ok) break;
            if (at == VT_STR) {
                for (uint64_t j = 0; ok && j < n; j++) {
                    std::string s;
                    ok = c.str(&s);
                }
            } else {
                if (n > (len_ - c.pos) / 4) ok = false;
                else c.pos += (size_t)n * 4;
            }
            break;
        }
        }
        if (!ok) {
            err = "Unexpected EOF reading metadata value";
            return NEXUS_E_TRUNCATED;
        }
        kv_[key] = v;
    }
    for (uint64_t t = 0; t < tc; t++) {
        GgufTensor ti;
        uint32_t nd, ty;
        if (!c.str(&ti.name) || !c.u32(&nd)) {
            err = "Unexpected EOF reading tensor info";
            return NEXUS_E_TRUNCATED;
        }
        if (nd > 8) {
            err = "Too many tensor dims";
            return NEXUS_E_INVALID;
        }
        for (uint32_t k = 0; k < nd; k++) {
            uint64_t dim;
            if (!c.u64(&dim)) {
                err = "Unexpected EOF reading shape";
                return NEXUS_E_TRUNCATED;
            }
            ti.shape.push_back(dim);
        }
        if (!c.u32(&ty) || !c.u64(&ti.offset)) {
            err = "Unexpected EOF reading tensor type/offset";
            return NEXUS_E_TRUNCATED;
        }
        ti.type = (int)ty;
        tensors_.push_back(ti);
    }
    auto it = kv_.find("general.alignment");
    if (it != kv_.end() && (it->second.vtype == VT_U32 || it->second.vtype == VT_U64))
        alignment_ = it->second.u;
    if (alignment_ < 1) alignment_ = 1;
    data_offset_ = (c.pos + alignment_ - 1) / alignment_ * alignment_;
    return NEXUS_OK;
}

const GgufTensor *GgufFile::find(const std::string &name) const {
    for (const auto &t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

const uint8_t *GgufFile::data(const GgufTensor &t, size_t *nbytes) const {
    if (!format_supported(t.type)) return nullptr;
    size_t n = format_bytes(t.type, t.elems());
    uint64_t off = data_offset_ + t.offset;
    if (off > len_ || n > len_ - off) return nullptr;
    if (nbytes) *nbytes = n;
    return map_ + off;
}

bool GgufFile::get_usize(const std::string &key, uint64_t *out) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return false;
    const GgufValue &v = it->second;
    if (v.vtype == VT_U64 || v.vtype == VT_U32) {
        *out = v.u;
        return true;
    }
    if ((v.vtype == VT_I64 || v.vtype == VT_I32) && v.i >= 0) {
        *out = (uint64_t)v.i;
        return true;
    }
    return false;
}

bool GgufFile::get_f32(const std::string &key, float *out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.vtype != VT_F32) return false;
    *out = (float)it->second.f;
    return true;
}

// ---------------------------------------------------------------------------
// host quantizer
// ---------------------------------------------------------------------------
size_t quantize_host(int fmt, const float *x, size_t n, uint8_t *out) {
    switch (fmt) {
    case F32: memcpy(out, x, n * 4); return n * 4;
    case F16:
        for (size_t i = 0; i < n; i++) st_f16(out + 2 * i, x[i]);
        return n * 2;
    case BF16: return 0;
    case Q8_0: case Q4_0: case Q4_K: case Q2_K: {
        size_t be = (size_t)block_elems(fmt), bb = (size_t)block_bytes(fmt), o = 0;
        float block[256];
        for (size_t c = 0; c < n; c += be, o += bb) {
            size_t len = std::min(be, n - c);
            memset(block, 0, sizeof(block));
            memcpy(block, x + c, len * sizeof(float));
            if (fmt == Q8_0) quantize_block_q8_0(block, (int)len, out + o);
            else if (fmt == Q4_0) quantize_block_q4_0(block, (int)len, out + o);
            else if (fmt == Q4_K) quantize_block_q4_k(block, out + o);
            else quantize_block_q2_k(block, out + o);
        }
        return o;
    }
    default: return 0;
    }
}

// ---------------------------------------------------------------------------
// synthetic model writer
// ---------------------------------------------------------------------------
// Counter-based normal generator: element i of tensor `stream` comes from pair
// p = i/2, r = splitmix64(splitmix64(seed ^ stream) + p); u1 = (r>>40 + 1)/2^24,
// u2 = (r & 0xffffff)/2^24; Box-Muller radius sqrt(-2 ln u1), angle 2*pi*u2;
// even i takes the cosine branch, odd i the sine branch.
static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}
static uint64_t fnv1a(const std::string &s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (unsigned char ch : s) {
        h ^= ch;
        h *= 0x100000001b3ull;
    }
    return h;
}
static void gen_normal(uint64_t seed, uint64_t stream, size_t start, size_t count, float stdv,
                       float *out) {
    uint64_t base = splitmix64(seed ^ stream);
    for (size_t k = 0; k < count; k++) {
        size_t i = start + k;
        uint64_t r = splitmix64(base + (uint64_t)(i / 2));
        float u1 = (float)((r >> 40) + 1) * (1.0f / 16777216.0f);
        float u2 = (float)(r & 0xffffffu) * (1.0f / 16777216.0f);
        float rad = sqrtf(-2.0f * logf(u1));
        float ang = 6.28318530717958647692f * u2;
        float z = (i & 1) ? rad * sinf(ang) : rad * cosf(ang);
        out[k] = stdv * z;
    }
}

struct SynthTensor {
    std::string name;
    std::vector<uint64_t> shape;
    int fmt;
    bool ones;
    size_t elems() const {
        size_t n = 1;
        for (auto d : shape) n *= (size_t)d;
        return n;
    }
};

static void put_u32(std::vector<uint8_t> &b, uint32_t v) {
    uint8_t t[4];
    memcpy(t, &v, 4);
    b.insert(b.end(), t, t + 4);
}
static void put_u64(std::vector<uint8_t> &b, uint64_t v) {
    uint8_t t[8];
    memcpy(t, &v, 8);
    b.insert(b.end(), t, t + 8);
}
static void put_str(std::vector<uint8_t> &b, const std::string &s) {
    put_u64(b, s.size());
    b.insert(b.end(), s.begin(), s.end());
}

int synth_model_write(const char *path, const nexus_synth_config *cfg, std::string &err) {
    const nexus_synth_config &C = *cfg;
    if (!C.num_layers && !C.hidden_size) {
        err = "empty config";
        return NEXUS_E_INVALID;
    }
    if (C.num_heads == 0 || C.hidden_size % C.num_heads) {
        err = "hidden_size must be a multiple of num_heads";
        return NEXUS_E_INVALID;
    }
    int fmts[] = {C.attn_format, C.ffn_format, C.embd_format, C.norm_format};
    for (int f : fmts)
        if (!format_supported(f) || f == BF16) {
            err = "unsupported synthetic format";
            return NEXUS_E_UNSUPPORTED_FORMAT;
        }
    if (C.head_format >= 0 && (!format_supported(C.head_format) || C.head_format == BF16)) {
        err = "unsupported head format";
        return NEXUS_E_UNSUPPORTED_FORMAT;
    }
    uint64_t H = C.hidden_size, F = C.ff_dim, V = C.vocab_size;
    uint64_t D = H / C.num_heads, KV = (uint64_t)C.num_kv_heads * D;
    std::vector<SynthTensor> ts;
    ts.push_back({"token_embd.weight", {V, H}, C.embd_format, false});
    ts.push_back({"output_norm.weight", {H}, C.norm_format, true});
    if (C.head_format >= 0) ts.push_back({"output.weight", {V, H}, C.head_format, false});
    for (uint32_t l = 0; l < C.num_layers; l++) {
        std::string p = "blk." + std::to_string(l) + ".";
        ts.push_back({p + "attn_norm.weight", {H}, C.norm_format, true});
        ts.push_back({p + "attn_q.weight", {H, H}, C.attn_format, false});
        ts.push_back({p + "attn_k.weight", {KV, H}, C.attn_format, false});
        ts.push_back({p + "attn_v.weight", {KV, H}, C.attn_format, false});
        ts.push_back({p + "attn_output.weight", {H, H}, C.attn_format, false});
        ts.push_back({p + "ffn_norm.weight", {H}, C.norm_format, true});
        ts.push_back({p + "ffn_gate.weight", {F, H}, C.ffn_format, false});
        ts.push_back({p + "ffn_up.weight", {F, H}, C.ffn_format, false});
        ts.push_back({p + "ffn_down.weight", {H, F}, C.ffn_format, false});
    }
    std::sort(ts.begin(), ts.end(), [](const SynthTensor &a, const SynthTensor &b) { return a.name < b.name; });

    const uint64_t ALIGN = 32;
    std::vector<uint8_t> hdr;
    hdr.insert(hdr.end(), {'G', 'G', 'U', 'F'});
    put_u32(hdr, 3);
    put_u64(hdr, ts.size());
    // metadata, sorted by key (tools/nexus-convert/main.rs:358-363)
    struct Kv { std::string key; int vt; uint32_t u; float f; std::string s; };
    std::vector<Kv> kvs = {
        {"general.alignment", VT_U32, (uint32_t)ALIGN, 0, ""},
        {"general.architecture", VT_STR, 0, 0, "llama"},
        {"general.name", VT_STR, 0, 0, "nexus-synthetic"},
        {"llama.attention.head_count", VT_U32, C.num_heads, 0, ""},
        {"llama.attention.head_count_kv", VT_U32, C.num_kv_heads, 0, ""},
        {"llama.attention.layer_norm_rms_epsilon", VT_F32, 0, 1e-5f, ""},
        {"llama.block_count", VT_U32, C.num_layers, 0, ""},
        {"llama.context_length", VT_U32, C.context_length, 0, ""},
        {"llama.embedding_length", VT_U32, C.hidden_size, 0, ""},
        {"llama.feed_forward_length", VT_U32, C.ff_dim, 0, ""},
        {"llama.rope.freq_base", VT_F32, 0, C.rope_theta, ""},
        {"llama.vocab_size", VT_U32, C.vocab_size, 0, ""},
    };
    std::sort(kvs.begin(), kvs.end(), [](const Kv &a, const Kv &b) { return a.key < b.key; });
    put_u64(hdr, kvs.size());
    for (auto &kv : kvs) {
        put_str(hdr, kv.key);
        put_u32(hdr, (uint32_t)kv.vt);
        if (kv.vt == VT_U32) put_u32(hdr, kv.u);
        else if (kv.vt == VT_F32) put_u32(hdr, f2u(kv.f));
        else put_str(hdr, kv.s);
    }
    uint64_t off = 0;
    std::vector<uint64_t> offsets, sizes;
    for (auto &t : ts) {
        put_str(hdr, t.name);
        put_u32(hdr, (uint32_t)t.shape.size());
        for (auto d : t.shape) put_u64(hdr, d);
        put_u32(hdr, (uint32_t)t.fmt);
        put_u64(hdr, off);
        uint64_t n = format_bytes(t.fmt, t.elems());
        offsets.push_back(off);
        sizes.push_back(n);
        off += (n + ALIGN - 1) / ALIGN * ALIGN;
    }
    while (hdr.size() % ALIGN) hdr.push_back(0);

    FILE *fp = fopen(path, "wb");
    if (!fp) {
        err = std::string("cannot create ") + path;
        return NEXUS_E_IO;
    }
    bool ok = fwrite(hdr.data(), 1, hdr.size(), fp) == hdr.size();
    int threads = C.threads > 0 ? C.threads : (int)std::max(1u, std::thread::hardware_concurrency());
    std::vector<uint8_t> buf;
    for (size_t ti = 0; ok && ti < ts.size(); ti++) {
        const SynthTensor &t = ts[ti];
        size_t n = t.elems();
        buf.assign((sizes[ti] + ALIGN - 1) / ALIGN * ALIGN, 0);
        uint64_t stream = fnv1a(t.name);
        // chunks of 64 Ki elements (a multiple of every block size)
        const size_t CH = 65536;
        size_t nchunks = (n + CH - 1) / CH;
        size_t be = (size_t)block_elems(t.fmt), bb = (size_t)block_bytes(t.fmt);
        // drawn chunks; with repeat_chunks the rest copy them (a whole chunk
        // is whole blocks, so its quantized bytes repeat exactly)
        const size_t drawn = C.repeat_chunks ? std::min<size_t>(nchunks, C.repeat_chunks) : nchunks;
        auto work = [&](int tid) {
            std::vector<float> vals(CH);
            for (size_t c = (size_t)tid; c < drawn; c += (size_t)threads) {
                size_t s = c * CH, cnt = std::min(CH, n - s);
                if (t.ones) std::fill(vals.begin(), vals.begin() + cnt, 1.0f);
                else gen_normal(C.seed, stream, s, cnt, C.weight_std, vals.data());
                quantize_host(t.fmt, vals.data(), cnt, buf.data() + s / be * bb);
            }
        };
        int nt = (int)std::min<size_t>((size_t)threads, drawn);
        if (nt <= 1) {
            work(0);
        } else {
            std::vector<std::thread> pool;
            for (int k = 0; k < nt; k++) pool.emplace_back(work, k);
            for (auto &th : pool) th.join();
        }
        for (size_t c = drawn; c < nchunks; c++) {
            const size_t s = c * CH, cnt = std::min(CH, n - s), src = (c % drawn) * CH;
            memcpy(buf.data() + s / be * bb, buf.data() + src / be * bb, cnt / be * bb);
        }
        ok = fwrite(buf.data(), 1, buf.size(), fp) == buf.size();
    }
    if (fclose(fp) != 0) ok = false;
    if (!ok) {
        err = std::string("write failed: ") + path;
        return NEXUS_E_IO;
    }
    return NEXUS_OK;
}

}  // namespace nx

extern "C" size_t nexus_quantize_host(int format, const float *x, size_t n, uint8_t *out) {
    return nx::quantize_host(format, x, n, out);
}

extern "C" size_t nexus_format_bytes(int format, size_t n) {
    if (!nx::format_supported(format)) return 0;
    return nx::format_bytes(format, n);
}
