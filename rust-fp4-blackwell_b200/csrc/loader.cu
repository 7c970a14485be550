// loader.cu -- real-weight checkpoints: a safetensors file with Hugging Face Llama
// tensor names, read on the host and quantised to MXFP4 on the GPU straight into
// the engine's layouts (and into this rank's shard under tensor parallelism).
//
// Replaces the reference's weight path (examples/llama_run/src/main.rs:413-460:
// safetensors loaded on the host, bf16/f16 widened to f32 (:425-427, :591-614),
// every linear quantised on the host by quant_fp4 (:334-376)).  Here the raw
// tensor bytes are copied to the device, widened there, and quantised with the
// E8M0 rule of the native format (the same quantiser as fp4_quantize_mxfp4,
// bit for bit) through the row maps the decode kernels read (rope-paired q/k
// tiles, gate/up interleaved by 8 rows).
//
// The safetensors format: 8-byte little-endian header length, a JSON object
// {"name": {"dtype": "BF16", "shape": [r, c], "data_offsets": [b, e]}, ...,
//  "__metadata__": {...}}, then the tensor bytes (offsets relative to the end of
// the header).  Supported dtypes: F32, BF16, F16.
#include "common.cuh"

#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace fp4x {
namespace loader {

struct Entry {
    int dtype = -1;  // 0 F32, 1 BF16, 2 F16
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;
};

// Recursive-descent reader for the header (strings, integers, arrays, objects).
struct Json {
    const char *p, *e;
    bool ok = true;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool take(char c) {
        ws();
        if (p < e && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    std::string str() {
        std::string s;
        if (!take('"')) {
            ok = false;
            return s;
        }
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) {
                ++p;
                if (*p == 'u') {  // names are ASCII; keep the escape verbatim
                    s += "\\u";
                    ++p;
                    continue;
                }
            }
            s += *p++;
        }
        if (p >= e) ok = false;
        ++p;
        return s;
    }
    bool integer(uint64_t &v) {
        ws();
        if (p >= e || *p < '0' || *p > '9') return false;
        v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (UINT64_MAX - 9) / 10) return ok = false;
            v = v * 10 + (uint64_t)(*p++ - '0');
        }
        return true;
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
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            ++p;
            if (take(close)) return;
            do {
                if (obj) {
                    str();
                    if (!take(':')) ok = false;
                }
                skip();
            } while (ok && take(','));
            if (!take(close)) ok = false;
        } else {
            while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;  // number / true / false / null
        }
    }
    bool int_array(std::vector<uint64_t> &out) {
        if (!take('[')) return false;
        if (take(']')) return true;
        do {
            uint64_t v;
            if (!integer(v)) return ok = false;
            out.push_back(v);
        } while (take(','));
        return take(']');
    }
};

int dtype_of(const std::string &d) { return d == "F32" ? 0 : d == "BF16" ? 1 : d == "F16" ? 2 : -1; }
size_t dtype_bytes(int d) { return d == 0 ? 4 : 2; }

struct File {
    FILE *f = nullptr;
    uint64_t data0 = 0, size = 0;
    std::map<std::string, Entry> t;
    ~File() {
        if (f) fclose(f);
    }
};

int open_file(const char *path, File &F) {
    FP4X_REQUIRE(path, "safetensors: null path");
    F.f = fopen(path, "rb");
    FP4X_REQUIRE(F.f, "safetensors: cannot open %s", path);
    fseek(F.f, 0, SEEK_END);
    F.size = (uint64_t)ftell(F.f);
    fseek(F.f, 0, SEEK_SET);
    uint8_t hl[8];
    FP4X_REQUIRE(F.size >= 8 && fread(hl, 1, 8, F.f) == 8, "safetensors: %s is too short", path);
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | hl[i];
    FP4X_REQUIRE(n >= 2 && n <= (1ull << 30) && 8 + n <= F.size, "safetensors: bad header length %llu in %s",
                 (unsigned long long)n, path);
    std::string h(n, '\0');
    FP4X_REQUIRE(fread(&h[0], 1, n, F.f) == n, "safetensors: short read of the header of %s", path);
    F.data0 = 8 + n;
    Json J{h.data(), h.data() + h.size()};
    FP4X_REQUIRE(J.take('{'), "safetensors: header of %s is not a JSON object", path);
    if (!J.take('}')) {
        do {
            const std::string name = J.str();
            FP4X_REQUIRE(J.ok && J.take(':'), "safetensors: malformed header in %s", path);
            if (name == "__metadata__") {
                J.skip();
                continue;
            }
            FP4X_REQUIRE(J.take('{'), "safetensors: tensor %s: expected an object", name.c_str());
            Entry en;
            bool have_off = false;
            if (!J.take('}')) {
                do {
                    const std::string key = J.str();
                    FP4X_REQUIRE(J.ok && J.take(':'), "safetensors: malformed entry %s", name.c_str());
                    if (key == "dtype") {
                        en.dtype = dtype_of(J.str());
                    } else if (key == "shape") {
                        FP4X_REQUIRE(J.int_array(en.shape), "safetensors: bad shape of %s", name.c_str());
                    } else if (key == "data_offsets") {
                        std::vector<uint64_t> o;
                        FP4X_REQUIRE(J.int_array(o) && o.size() == 2 && o[0] <= o[1],
                                     "safetensors: bad data_offsets of %s", name.c_str());
                        en.begin = o[0], en.end = o[1], have_off = true;
                    } else {
                        J.skip();
                    }
                } while (J.ok && J.take(','));
                FP4X_REQUIRE(J.ok && J.take('}'), "safetensors: malformed entry %s", name.c_str());
            }
            FP4X_REQUIRE(have_off, "safetensors: %s has no data_offsets", name.c_str());
            uint64_t count = 1;
            for (uint64_t d : en.shape) count *= d;
            if (en.dtype >= 0)
                FP4X_REQUIRE(en.end - en.begin == count * dtype_bytes(en.dtype) && F.data0 + en.end <= F.size,
                             "safetensors: %s: %llu bytes for its shape, or past the end of the file", name.c_str(),
                             (unsigned long long)(en.end - en.begin));
            F.t[name] = en;
        } while (J.ok && J.take(','));
        FP4X_REQUIRE(J.ok && J.take('}'), "safetensors: malformed header in %s", path);
    }
    return FP4X_OK;
}

// Tensor `name` with the given shape, widened to f32 into dev (device, >= count floats).
int read_f32(File &F, cudaStream_t st, const std::string &name, std::vector<uint64_t> shape, void *raw_dev,
             float *dev);

__global__ void widen_kernel(const void *raw, int dtype, size_t n, float *out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (dtype == 0) {
            out[i] = static_cast<const float *>(raw)[i];
        } else if (dtype == 1) {
            out[i] = __uint_as_float((uint32_t)static_cast<const uint16_t *>(raw)[i] << 16);
        } else {
            out[i] = __half2float(static_cast<const __half *>(raw)[i]);
        }
    }
}

__global__ void to_bf16_kernel(const float *x, size_t n, uint16_t *out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = f32_to_bf16_bits(x[i]);
}

// Rows [row0, row0 + n) and columns [col0, col0 + k) of the f32 [*][k_global]
// matrix src, quantised per 32-block (E8M0 rule) into rows map_row(r) of packed/scales.
__global__ void quant_rows_kernel(const float *__restrict__ src, uint32_t k_global, uint32_t n, uint32_t k,
                                  uint32_t row0, uint32_t col0, uint8_t *__restrict__ packed,
                                  uint8_t *__restrict__ scales, int mode, uint32_t off, uint32_t hd) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t nbr = k / 32;
    if (blk >= (uint64_t)n * nbr) return;
    const uint32_t r = (uint32_t)(blk / nbr), b = (uint32_t)(blk % nbr);
    const float *row = src + (size_t)(row0 + r) * k_global + col0 + 32u * b;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = row[i];
    uint4 p;
    uint8_t s;
    quant::quant_block_mxfp4(v, p, s);
    const uint64_t dblk = (uint64_t)quant::map_row(r, mode, off, hd) * nbr + b;
    reinterpret_cast<uint4 *>(packed)[dblk] = p;
    scales[dblk] = s;
}

int read_f32(File &F, cudaStream_t st, const std::string &name, std::vector<uint64_t> shape, void *raw_dev,
             float *dev) {
    auto it = F.t.find(name);
    FP4X_REQUIRE(it != F.t.end(), "safetensors: tensor %s not found", name.c_str());
    const Entry &en = it->second;
    FP4X_REQUIRE(en.dtype >= 0, "safetensors: %s has an unsupported dtype (F32, BF16, F16 are read)", name.c_str());
    FP4X_REQUIRE(en.shape == shape, "safetensors: %s has the wrong shape for this config", name.c_str());
    const size_t bytes = en.end - en.begin, count = bytes / dtype_bytes(en.dtype);
    std::vector<uint8_t> host(bytes);
    FP4X_REQUIRE(fseek(F.f, (long)(F.data0 + en.begin), SEEK_SET) == 0 && fread(host.data(), 1, bytes, F.f) == bytes,
                 "safetensors: short read of %s", name.c_str());
    if (cudaMemcpyAsync(raw_dev, host.data(), bytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return engine::cuda_fail("safetensors: upload", cudaGetLastError());
    widen_kernel<<<(unsigned)std::min<size_t>((count + 255) / 256, 4096), 256, 0, st>>>(raw_dev, en.dtype, count, dev);
    if (int e = check_launch("safetensors: widen")) return e;
    if (cudaStreamSynchronize(st) != cudaSuccess) return engine::cuda_fail("safetensors: widen", cudaGetLastError());
    return FP4X_OK;
}

int quant_into(cudaStream_t st, const float *src, uint32_t k_global, uint32_t n, uint32_t k, uint32_t row0,
               uint32_t col0, uint8_t *packed, uint8_t *scales, int mode, uint32_t off, uint32_t hd) {
    const uint64_t nb = (uint64_t)n * (k / 32);
    quant_rows_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, st>>>(src, k_global, n, k, row0, col0, packed, scales,
                                                                     mode, off, hd);
    if (int e = check_launch("safetensors: quantise")) return e;
    if (cudaStreamSynchronize(st) != cudaSuccess) return engine::cuda_fail("safetensors: quantise", cudaGetLastError());
    return FP4X_OK;
}

}  // namespace loader

namespace engine {

// The model's weights from a checkpoint instead of the seeded generator (the
// counterpart of init_weights; same shards, same layouts).
int load_safetensors(fp4x_llama_model *m, cudaStream_t st, const char *path) {
    using loader::File;
    File F;
    FP4X_TRY(loader::open_file(path, F));
    const fp4x_llama_config &c = m->lc, &g = m->cfg;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd, r = g.tp_size > 1 ? g.tp_rank : 0;
    const uint64_t gqd = (uint64_t)g.n_heads * hd, gkvd = (uint64_t)g.n_kv_heads * hd;
    // staging: the largest tensor (embeddings / lm_head or an FFN matrix)
    const uint64_t most = std::max<uint64_t>({(uint64_t)g.vocab * g.dim, (uint64_t)g.ffn * g.dim, gqd * g.dim});
    void *raw = nullptr;
    float *f32 = nullptr;
    if (cudaMalloc(&raw, most * 4) != cudaSuccess || cudaMalloc(&f32, most * 4) != cudaSuccess) {
        if (raw) cudaFree(raw);
        set_error("safetensors: staging allocation of %llu bytes failed", (unsigned long long)(most * 8));
        return FP4X_ENOMEM;
    }
    auto rd = [&](const std::string &name, std::vector<uint64_t> shape) { return loader::read_f32(F, st, name, shape, raw, f32); };
    int rc = FP4X_OK;
    const uint64_t D = g.dim, FF = g.ffn;
    for (uint32_t l = 0; l < c.n_layers && !rc; ++l) {
        LayerW &L = m->layers[l];
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        rc = rd(pre + "self_attn.q_proj.weight", {gqd, D});
        if (!rc) rc = loader::quant_into(st, f32, g.dim, qd, c.dim, r * qd, 0, L.qkv.w, L.qkv.s, 1, 0, hd);
        if (!rc) rc = rd(pre + "self_attn.k_proj.weight", {gkvd, D});
        if (!rc) rc = loader::quant_into(st, f32, g.dim, kvd, c.dim, r * kvd, 0, L.qkv.w, L.qkv.s, 1, qd, hd);
        if (!rc) rc = rd(pre + "self_attn.v_proj.weight", {gkvd, D});
        if (!rc) rc = loader::quant_into(st, f32, g.dim, kvd, c.dim, r * kvd, 0, L.qkv.w, L.qkv.s, 0, qd + kvd, hd);
        if (!rc) rc = rd(pre + "self_attn.o_proj.weight", {D, gqd});
        if (!rc) rc = loader::quant_into(st, f32, (uint32_t)gqd, c.dim, qd, 0, r * qd, L.o.w, L.o.s, 0, 0, hd);
        if (!rc) rc = rd(pre + "mlp.gate_proj.weight", {FF, D});
        if (!rc) rc = loader::quant_into(st, f32, g.dim, c.ffn, c.dim, r * c.ffn, 0, L.gu.w, L.gu.s, 2, 0, hd);
        if (!rc) rc = rd(pre + "mlp.up_proj.weight", {FF, D});
        if (!rc) rc = loader::quant_into(st, f32, g.dim, c.ffn, c.dim, r * c.ffn, 0, L.gu.w, L.gu.s, 2, 8, hd);
        if (!rc) rc = rd(pre + "mlp.down_proj.weight", {D, FF});
        if (!rc) rc = loader::quant_into(st, f32, g.ffn, c.dim, c.ffn, 0, r * c.ffn, L.down.w, L.down.s, 0, 0, hd);
        if (!rc) rc = rd(pre + "input_layernorm.weight", {D});
        if (!rc && cudaMemcpyAsync(L.attn_norm, f32, D * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            rc = cuda_fail("safetensors: norm", cudaGetLastError());
        if (!rc) rc = rd(pre + "post_attention_layernorm.weight", {D});
        if (!rc && cudaMemcpyAsync(L.ffn_norm, f32, D * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            rc = cuda_fail("safetensors: norm", cudaGetLastError());
        if (!rc && (cudaMemsetAsync(L.kc, 0, (size_t)c.max_seq * kvd * 2, st) != cudaSuccess ||
                    cudaMemsetAsync(L.vc, 0, (size_t)c.max_seq * kvd * 2, st) != cudaSuccess))
            rc = cuda_fail("safetensors: KV clear", cudaGetLastError());
    }
    if (!rc) rc = rd("model.norm.weight", {D});
    if (!rc && (cudaMemcpyAsync(m->final_norm, f32, D * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess))
        rc = cuda_fail("safetensors: final norm", cudaGetLastError());
    if (!rc) rc = rd("model.embed_tokens.weight", {(uint64_t)g.vocab, D});
    if (!rc) {
        const size_t n = (size_t)g.vocab * g.dim;
        loader::to_bf16_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, st>>>(f32, n, m->embed);
        rc = check_launch("safetensors: embeddings");
        if (!rc && cudaStreamSynchronize(st) != cudaSuccess) rc = cuda_fail("safetensors: embeddings", cudaGetLastError());
    }
    // lm_head, or the embeddings when the checkpoint ties them
    if (!rc) rc = rd(F.t.count("lm_head.weight") ? "lm_head.weight" : "model.embed_tokens.weight", {(uint64_t)g.vocab, D});
    if (!rc) rc = loader::quant_into(st, f32, g.dim, c.vocab, c.dim, m->v0, 0, m->lm_head.w, m->lm_head.s, 0, 0, hd);
    if (!rc) rc = llama_rope_tables((fp4x_stream_t)st, c.max_seq, hd, (double)c.rope_theta, m->cos_t, m->sin_t);
    cudaStreamSynchronize(st);
    cudaFree(raw);
    cudaFree(f32);
    return rc;
}

}  // namespace engine
}  // namespace fp4x

using namespace fp4x;

extern "C" int fp4x_safetensors_info(const char *path, const char *name, uint32_t *dtype_out, uint64_t *shape_out,
                                     uint32_t *ndim_out) {
    FP4X_REQUIRE(name, "fp4x_safetensors_info: null name");
    loader::File F;
    FP4X_TRY(loader::open_file(path, F));
    auto it = F.t.find(name);
    FP4X_REQUIRE(it != F.t.end(), "safetensors: tensor %s not found in %s", name, path);
    if (dtype_out) *dtype_out = (uint32_t)it->second.dtype;
    if (ndim_out) *ndim_out = (uint32_t)it->second.shape.size();
    if (shape_out)
        for (size_t i = 0; i < it->second.shape.size() && i < 8; ++i) shape_out[i] = it->second.shape[i];
    return FP4X_OK;
}

extern "C" int llama_model_create_from_safetensors(const fp4x_llama_config *cfg, const char *path,
                                                   fp4x_llama_model **out) {
    FP4X_REQUIRE(path, "llama_model_create_from_safetensors: null path");
    return engine::create(cfg, out, path);
}
