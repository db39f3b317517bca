// sme_loader.cu -- `.sme` model files and the int4 group-128 weight converter.
//
// Container (the reference's format, model/README.md:9-36; written by
// convert_model.py:26-67 save_sme_model, read by server/main.cpp:112-228
// load_sme_model):
//   "SME_MODEL" | u32 config_len | config JSON | u32 n_vocab | n_vocab x (u32 len,
//   bytes) | u32 n_tensors | n_tensors x (u32 name_len, name | u32 n_dims,
//   u32 dims[n_dims] | u8 quantized | u32 data_size | quantized: f32
//   row_scale[dims[0]], int8 data[prod dims]; else f32 data[prod dims]).
// Offsets advance by the element count (prod dims), not by data_size, as in
// main.cpp:207-221; every field is bounds-checked against the file size and a
// short or malformed file is SPECDEC_EFORMAT.  A later tensor with the name of
// an earlier one replaces it (main.cpp:222, map assignment).
//
// int8 rows carry the writer's row factor rs = 127 / max|w| and
// q = round(w * rs) (convert_model.py:8-23), so the weight is q / rs -- the
// formula of model/README.md:41-52.  (The reference forward multiplies by rs
// instead, server/sme_gemm.cpp:16-36; it also reads embed_tokens as f32 although
// the writer stores it as int8 rows.  Both are reference defects; the loader
// follows the writer.)
//
// The converter turns int8 (or f32) rows into the library's W4A16 tiled units
// on the device: one warp per (row, 128-column group) forms the group's values
// (q / rs, times an optional per-column RMSNorm weight folded in), takes
// amax, s = fp16(amax / 7) (1 when amax = 0), q4 = clamp(round(v / s), -8, 7)
// and writes the group's 16 nibble words and its scale straight into the
// 8448-byte unit -- the same quantiser as the synthetic-weight generator.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "internal.h"

struct specdec_sme {
    const uint8_t* base = nullptr;
    size_t size = 0;
    void* map = nullptr;  // mmap'd file (nullptr for a caller-owned buffer)
    size_t map_size = 0;
    std::string config;
    std::vector<std::pair<size_t, uint32_t>> vocab;  // (offset, length) of each token
    std::unordered_map<std::string, int32_t> token_id;
    struct Tensor {
        std::string name;
        std::vector<uint32_t> dims;
        uint64_t elements;
        uint8_t quantized;
        uint32_t data_bytes;
        size_t scales_off;  // quantized: offset of f32 row scales
        size_t data_off;
    };
    std::vector<Tensor> tensors;  // in file order, replaced names removed
    std::unordered_map<std::string, size_t> by_name;
};

namespace specdec {
namespace {

struct Cursor {
    const uint8_t* p;
    size_t n, at = 0;
    bool take(size_t bytes) {
        if (bytes > n - at) return false;
        at += bytes;
        return true;
    }
    bool u32(uint32_t* v) {
        if (4 > n - at) return false;
        std::memcpy(v, p + at, 4);
        at += 4;
        return true;
    }
};

int parse(specdec_sme* f) {
    Cursor c{f->base, f->size};
    SD_CHECK(f->size >= 9 && std::memcmp(f->base, "SME_MODEL", 9) == 0, SPECDEC_EFORMAT,
             "sme: magic header mismatch");
    c.at = 9;
    uint32_t cfg_len = 0;
    SD_CHECK(c.u32(&cfg_len) && cfg_len <= c.n - c.at, SPECDEC_EFORMAT, "sme: truncated config");
    f->config.assign(reinterpret_cast<const char*>(f->base + c.at), cfg_len);
    c.at += cfg_len;
    uint32_t nv = 0;
    SD_CHECK(c.u32(&nv), SPECDEC_EFORMAT, "sme: truncated vocabulary size");
    SD_CHECK((uint64_t)nv * 4 <= c.n - c.at, SPECDEC_EFORMAT, "sme: truncated vocabulary");
    f->vocab.resize(nv);
    f->token_id.reserve(nv);
    for (uint32_t i = 0; i < nv; ++i) {
        uint32_t len = 0;
        SD_CHECK(c.u32(&len), SPECDEC_EFORMAT, "sme: truncated token length");
        const size_t off = c.at;
        SD_CHECK(c.take(len), SPECDEC_EFORMAT, "sme: truncated token");
        f->vocab[i] = {off, len};
        f->token_id[std::string(reinterpret_cast<const char*>(f->base + off), len)] = (int32_t)i;
    }
    uint32_t nt = 0;
    SD_CHECK(c.u32(&nt), SPECDEC_EFORMAT, "sme: truncated tensor count");
    for (uint32_t t = 0; t < nt; ++t) {
        specdec_sme::Tensor T;
        uint32_t nl = 0;
        SD_CHECK(c.u32(&nl), SPECDEC_EFORMAT, "sme: truncated tensor name length");
        SD_CHECK(nl <= c.n - c.at, SPECDEC_EFORMAT, "sme: truncated tensor name");
        T.name.assign(reinterpret_cast<const char*>(f->base + c.at), nl);
        c.at += nl;
        uint32_t nd = 0;
        SD_CHECK(c.u32(&nd), SPECDEC_EFORMAT, "sme: truncated dimension count");
        SD_CHECK((uint64_t)nd * 4 <= c.n - c.at, SPECDEC_EFORMAT, "sme: truncated dimensions");
        T.dims.resize(nd);
        T.elements = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            c.u32(&T.dims[d]);
            SD_CHECK(T.dims[d] == 0 || T.elements <= (uint64_t)f->size / T.dims[d], SPECDEC_EFORMAT,
                     "sme: tensor larger than the file");
            T.elements *= T.dims[d];
        }
        SD_CHECK(c.at < c.n, SPECDEC_EFORMAT, "sme: truncated quantisation flag");
        T.quantized = f->base[c.at++] == 1 ? 1 : 0;
        SD_CHECK(c.u32(&T.data_bytes), SPECDEC_EFORMAT, "sme: truncated data size");
        T.scales_off = c.at;
        if (T.quantized) {
            SD_CHECK(nd >= 1, SPECDEC_EFORMAT, "sme: quantised tensor without dimensions");
            SD_CHECK(c.take((size_t)T.dims[0] * 4), SPECDEC_EFORMAT, "sme: truncated row scales");
            T.data_off = c.at;
            SD_CHECK(c.take((size_t)T.elements), SPECDEC_EFORMAT, "sme: truncated int8 data");
        } else {
            T.data_off = c.at;
            SD_CHECK(T.elements <= (c.n - c.at) / 4 && c.take((size_t)T.elements * 4), SPECDEC_EFORMAT,
                     "sme: truncated f32 data");
        }
        auto it = f->by_name.find(T.name);
        if (it != f->by_name.end()) {
            f->tensors[it->second] = std::move(T);
        } else {
            f->by_name.emplace(T.name, f->tensors.size());
            f->tensors.push_back(std::move(T));
        }
    }
    return SPECDEC_OK;
}

void fill_view(const specdec_sme* f, const specdec_sme::Tensor& t, specdec_sme_tensor* out) {
    out->name = t.name.c_str();
    out->n_dims = (uint32_t)t.dims.size();
    out->dims = t.dims.data();
    out->elements = t.elements;
    out->quantized = t.quantized;
    out->data_bytes = t.data_bytes;
    out->scales = t.quantized ? f->base + t.scales_off : nullptr;
    out->data = f->base + t.data_off;
}

// Value of a top-level JSON key: the text after `"key"` and its colon, as
// the reference's extract_int does (main.cpp:129-135), parsed as a number.
bool config_number(const std::string& cfg, const char* key, double* out) {
    const std::string k = std::string("\"") + key + "\"";
    size_t pos = cfg.find(k);
    if (pos == std::string::npos) return false;
    pos = cfg.find(':', pos + k.size());
    if (pos == std::string::npos) return false;
    const char* s = cfg.c_str() + pos + 1;
    char* end = nullptr;
    const double v = std::strtod(s, &end);
    if (end == s) return false;
    *out = v;
    return true;
}

}  // namespace

const specdec_sme::Tensor* sme_find(const specdec_sme* f, const std::string& name) {
    auto it = f->by_name.find(name);
    return it == f->by_name.end() ? nullptr : &f->tensors[it->second];
}

// Tensor of a role under the reference's short names (convert_model.py:79-97,
// read at main.cpp:262-352) or, failing that, under the Hugging Face names that
// convert_model.py's checkpoint path writes (model.named_parameters()).
const specdec_sme::Tensor* sme_role(const specdec_sme* f, const char* role, int layer) {
    static const struct {
        const char* role;
        const char* ref;
        const char* hf;
    } kNames[] = {
        {"embed", "embed_tokens", "model.embed_tokens.weight"},
        {"norm", "norm", "model.norm.weight"},
        {"lm_head", "lm_head", "lm_head.weight"},
        {"q", "layers.%d.q_proj", "model.layers.%d.self_attn.q_proj.weight"},
        {"k", "layers.%d.k_proj", "model.layers.%d.self_attn.k_proj.weight"},
        {"v", "layers.%d.v_proj", "model.layers.%d.self_attn.v_proj.weight"},
        {"o", "layers.%d.o_proj", "model.layers.%d.self_attn.o_proj.weight"},
        {"gate", "layers.%d.gate_proj", "model.layers.%d.mlp.gate_proj.weight"},
        {"up", "layers.%d.up_proj", "model.layers.%d.mlp.up_proj.weight"},
        {"down", "layers.%d.down_proj", "model.layers.%d.mlp.down_proj.weight"},
        {"attn_norm", "layers.%d.attn_norm", "model.layers.%d.input_layernorm.weight"},
        {"ffn_norm", "layers.%d.ffn_norm", "model.layers.%d.post_attention_layernorm.weight"},
        {"mtp", "mtp.%d.proj", "mtp.%d.proj.weight"},
        {"mtp_norm", "mtp.%d.norm", "mtp.%d.norm.weight"},
    };
    for (const auto& n : kNames) {
        if (std::strcmp(n.role, role) != 0) continue;
        char buf[128];
        for (const char* pat : {n.ref, n.hf}) {
            std::snprintf(buf, sizeof(buf), pat, layer);
            if (const auto* t = sme_find(f, buf)) return t;
        }
        return nullptr;
    }
    return nullptr;
}

bool sme_role_view(const specdec_sme* f, const char* role, int layer, specdec_sme_tensor* out) {
    const auto* t = sme_role(f, role, layer);
    if (t) fill_view(f, *t, out);
    return t != nullptr;
}

// --------------------------------------------------------------- converter
__device__ __forceinline__ float w4_source_value(const W4Source& s, int r, int t) {
    float v;
    if (s.q8) {
        v = __fdiv_rn((float)s.q8[(size_t)r * s.K + t], s.rs[r]);
    } else {
        v = s.f32[(size_t)r * s.K + t];
    }
    if (s.fold) v = __fmul_rn(v, s.fold[t]);
    return v;
}

// Destination row of source row r: row0 + r (layout 0), or the gate (1) / up
// (2) half of the fused SwiGLU weight, whose 256-row tile t holds gate rows
// 128t .. 128t+127 then the up rows of the same features.
__device__ __forceinline__ int w4_dest_row(int r, int row0, int layout) {
    if (layout == 0) return row0 + r;
    return ((r >> 7) << 8) + (layout == 2 ? 128 : 0) + (r & 127);
}

__global__ void __launch_bounds__(256) w4_convert_kernel(W4Source src, int rows, int row0, int layout, int KG,
                                                         uint8_t* __restrict__ tiled) {
    const int lane = threadIdx.x & 31;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t wi = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wi < (size_t)rows * KG;
         wi += warps) {
        const int r = (int)(wi / KG), g = (int)(wi % KG);
        const int t0 = g * 128 + 4 * lane;
        float v[4];
        float amax = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            v[m] = t0 + m < src.K ? w4_source_value(src, r, t0 + m) : 0.f;
            amax = fmaxf(amax, fabsf(v[m]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        __half s16 = __float2half_rn(__fdiv_rn(amax, 7.0f));
        if (amax == 0.f) s16 = __float2half_rn(1.0f);
        const float sf = __half2float(s16);
        // lane holds k = 4 lane + m of the group: word kc = lane / 2, element
        // i = 4 (lane & 1) + m, nibble j = i / 2 (even i) or j + 4 (odd i)
        uint32_t part = 0;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            uint32_t u = 8;
            if (t0 + m < src.K) {
                int q = (int)roundf(__fdiv_rn(v[m], sf));
                q = q < -8 ? -8 : (q > 7 ? 7 : q);
                u = (uint32_t)(q + 8);
            }
            const int i = 4 * (lane & 1) + m, j = i >> 1;
            part |= u << ((i & 1) ? (4 * j + 16) : (4 * j));
        }
        part |= __shfl_xor_sync(0xffffffffu, part, 1);
        const int n = w4_dest_row(r, row0, layout);
        uint8_t* unit = tiled + ((size_t)(n >> 7) * KG + g) * 8448;
        if (!(lane & 1)) *reinterpret_cast<uint32_t*>(unit + (((lane >> 1) * 128 + (n & 127)) << 2)) = part;
        if (lane == 0) *reinterpret_cast<__half*>(unit + 8192 + (n & 127) * 2) = s16;
    }
}

// Every unit to weight zero: nibbles 8, scales 0 (padding rows and columns).
__global__ void w4_fill_zero_kernel(uint32_t* __restrict__ tiled, size_t units) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < units * 2112; i += (size_t)gridDim.x * blockDim.x)
        tiled[i] = (i % 2112) < 2048 ? 0x88888888u : 0u;
}

__global__ void f16_rows_kernel(W4Source src, int rows, __half* __restrict__ out) {
    const size_t n = (size_t)rows * src.K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(w4_source_value(src, (int)(i / src.K), (int)(i % src.K)));
}

int w4_convert_launch(const W4Source& src, int rows, int row0, int layout, uint8_t* tiled, int KG, cudaStream_t s) {
    if (rows <= 0) return SPECDEC_OK;
    const size_t warps = (size_t)rows * KG;
    const unsigned blocks = (unsigned)std::min<size_t>((warps + 7) / 8, 148u * 16u);
    w4_convert_kernel<<<blocks, 256, 0, s>>>(src, rows, row0, layout, KG, tiled);
    SD_LAUNCH_CHECK("w4_convert_kernel");
    return SPECDEC_OK;
}

int w4_fill_zero_launch(uint8_t* tiled, size_t units, cudaStream_t s) {
    if (!units) return SPECDEC_OK;
    w4_fill_zero_kernel<<<148 * 8, 256, 0, s>>>(reinterpret_cast<uint32_t*>(tiled), units);
    SD_LAUNCH_CHECK("w4_fill_zero_kernel");
    return SPECDEC_OK;
}

int f16_rows_launch(const W4Source& src, int rows, __half* out, cudaStream_t s) {
    if (rows <= 0) return SPECDEC_OK;
    f16_rows_kernel<<<148 * 8, 256, 0, s>>>(src, rows, out);
    SD_LAUNCH_CHECK("f16_rows_kernel");
    return SPECDEC_OK;
}

// Streams a file tensor's rows through a device staging buffer and converts
// them: to W4 tiled units (layout / row0 as w4_convert_launch) or, when f16 is
// given, to fp16 rows.  fold: device f32 [K] or null.  Chunks hold whole
// 128-row groups so gate / up chunks stay unit-aligned.
int sme_upload_convert(const specdec_sme_tensor& t, const float* fold, uint8_t* tiled, int KG, int row0, int layout,
                       __half* f16, uint8_t* stage, size_t stage_bytes, cudaStream_t s) {
    SD_CHECK(t.n_dims == 2 && t.dims[1] > 0 && t.dims[1] % 8 == 0, SPECDEC_EFORMAT,
             std::string("sme: ") + t.name + " must be 2-D with a multiple of 8 columns");
    const int rows = (int)t.dims[0], K = (int)t.dims[1];
    const size_t elem = t.quantized ? 1 : 4;
    const size_t row_bytes = (size_t)K * elem + (t.quantized ? 4 : 0);
    size_t chunk = (stage_bytes - 256) / row_bytes;
    chunk = chunk >= 128 ? chunk / 128 * 128 : chunk;
    chunk = std::min<size_t>(chunk, (size_t)rows);
    SD_CHECK(chunk > 0, SPECDEC_EINVAL, "sme: staging buffer smaller than one row");
    SD_CHECK(layout == 0 || f16 || chunk == (size_t)rows || chunk % 128 == 0, SPECDEC_EINVAL,
             "sme: gate/up chunk not 128-row aligned");
    const uint8_t* data = static_cast<const uint8_t*>(t.data);
    const uint8_t* scales = static_cast<const uint8_t*>(t.scales);
    for (int r0 = 0; r0 < rows; r0 += (int)chunk) {
        const int n = std::min((int)chunk, rows - r0);
        W4Source src{};
        src.K = K;
        src.fold = fold;
        const size_t data_bytes = (size_t)n * K * elem;
        const size_t sc_off = (data_bytes + 255) & ~(size_t)255;  // row factors after the data
        SD_CUDA(cudaMemcpyAsync(stage, data + (size_t)r0 * K * elem, data_bytes, cudaMemcpyHostToDevice, s));
        if (t.quantized) {
            SD_CUDA(cudaMemcpyAsync(stage + sc_off, scales + (size_t)r0 * 4, (size_t)n * 4, cudaMemcpyHostToDevice, s));
            src.q8 = reinterpret_cast<const int8_t*>(stage);
            src.rs = reinterpret_cast<const float*>(stage + sc_off);
        } else {
            src.f32 = reinterpret_cast<const float*>(stage);
        }
        int rc;
        if (f16) {
            rc = f16_rows_launch(src, n, f16 + (size_t)r0 * K, s);
        } else if (layout == 0) {
            rc = w4_convert_launch(src, n, row0 + r0, 0, tiled, KG, s);
        } else {
            rc = w4_convert_launch(src, n, 0, layout, tiled + (size_t)(r0 / 128) * 2 * KG * 8448, KG, s);
        }
        if (rc) return rc;
    }
    return SPECDEC_OK;
}

}  // namespace specdec

using namespace specdec;

extern "C" int specdec_sme_open_buffer(const void* data, size_t bytes, specdec_sme** out) {
    SD_CHECK(out && (data || !bytes), SPECDEC_EINVAL, "sme_open_buffer: null argument");
    *out = nullptr;
    specdec_sme* f = new specdec_sme();
    f->base = static_cast<const uint8_t*>(data);
    f->size = bytes;
    const int rc = parse(f);
    if (rc) {
        delete f;
        return rc;
    }
    *out = f;
    return SPECDEC_OK;
}

extern "C" int specdec_sme_open(const char* path, specdec_sme** out) {
    SD_CHECK(path && out, SPECDEC_EINVAL, "sme_open: null argument");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY);
    SD_CHECK(fd >= 0, SPECDEC_EIO, std::string("sme_open: cannot open ") + path);
    struct stat st {};
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        SD_CHECK(false, SPECDEC_EIO, "sme_open: fstat failed");
    }
    void* map = nullptr;
    if (st.st_size > 0) {
        map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) {
            ::close(fd);
            SD_CHECK(false, SPECDEC_EIO, "sme_open: mmap failed");
        }
    }
    ::close(fd);  // the mapping keeps the file
    specdec_sme* f = new specdec_sme();
    f->map = map;
    f->map_size = (size_t)st.st_size;
    f->base = static_cast<const uint8_t*>(map);
    f->size = (size_t)st.st_size;
    const int rc = parse(f);
    if (rc) {
        if (map) munmap(map, f->map_size);
        delete f;
        return rc;
    }
    *out = f;
    return SPECDEC_OK;
}

extern "C" int specdec_sme_close(specdec_sme* f) {
    if (!f) return SPECDEC_OK;
    if (f->map) munmap(f->map, f->map_size);
    delete f;
    return SPECDEC_OK;
}

extern "C" int specdec_sme_config_json(const specdec_sme* f, const char** json, size_t* len) {
    SD_CHECK(f && json && len, SPECDEC_EINVAL, "sme_config_json: null argument");
    *json = f->config.data();
    *len = f->config.size();
    return SPECDEC_OK;
}

extern "C" int specdec_sme_config_number(const specdec_sme* f, const char* key, double* value) {
    SD_CHECK(f && key && value, SPECDEC_EINVAL, "sme_config_number: null argument");
    SD_CHECK(config_number(f->config, key, value), SPECDEC_EINVAL, std::string("sme: config has no number ") + key);
    return SPECDEC_OK;
}

extern "C" int specdec_sme_vocab_size(const specdec_sme* f, uint32_t* n) {
    SD_CHECK(f && n, SPECDEC_EINVAL, "sme_vocab_size: null argument");
    *n = (uint32_t)f->vocab.size();
    return SPECDEC_OK;
}

extern "C" int specdec_sme_token(const specdec_sme* f, uint32_t id, const char** text, uint32_t* len) {
    SD_CHECK(f && text && len, SPECDEC_EINVAL, "sme_token: null argument");
    SD_CHECK(id < f->vocab.size(), SPECDEC_EINVAL, "sme_token: id out of range");
    *text = reinterpret_cast<const char*>(f->base + f->vocab[id].first);
    *len = f->vocab[id].second;
    return SPECDEC_OK;
}

extern "C" int specdec_sme_token_id(const specdec_sme* f, const char* text, uint32_t len, int32_t* id) {
    SD_CHECK(f && (text || !len) && id, SPECDEC_EINVAL, "sme_token_id: null argument");
    auto it = f->token_id.find(std::string(text ? text : "", len));
    *id = it == f->token_id.end() ? 1 : it->second;  // unknown word -> 1 (main.cpp:230-233)
    return SPECDEC_OK;
}

extern "C" int specdec_sme_tensor_count(const specdec_sme* f, uint32_t* n) {
    SD_CHECK(f && n, SPECDEC_EINVAL, "sme_tensor_count: null argument");
    *n = (uint32_t)f->tensors.size();
    return SPECDEC_OK;
}

extern "C" int specdec_sme_tensor_at(const specdec_sme* f, uint32_t index, specdec_sme_tensor* out) {
    SD_CHECK(f && out, SPECDEC_EINVAL, "sme_tensor_at: null argument");
    SD_CHECK(index < f->tensors.size(), SPECDEC_EINVAL, "sme_tensor_at: index out of range");
    fill_view(f, f->tensors[index], out);
    return SPECDEC_OK;
}

extern "C" int specdec_sme_find(const specdec_sme* f, const char* name, specdec_sme_tensor* out) {
    SD_CHECK(f && name && out, SPECDEC_EINVAL, "sme_find: null argument");
    const auto* t = sme_find(f, name);
    SD_CHECK(t, SPECDEC_EINVAL, std::string("sme: no tensor ") + name);
    fill_view(f, *t, out);
    return SPECDEC_OK;
}

extern "C" int specdec_sme_model_config(const specdec_sme* f, specdec_model_config* mc) {
    SD_CHECK(f && mc, SPECDEC_EINVAL, "sme_model_config: null argument");
    double v = 0;
    auto num = [&](const char* key, double dflt) { return config_number(f->config, key, &v) ? v : dflt; };
    const auto* emb = sme_role(f, "embed", 0);
    const auto* k0 = sme_role(f, "k", 0);
    const auto* g0 = sme_role(f, "gate", 0);
    SD_CHECK(emb && emb->dims.size() == 2 && k0 && k0->dims.size() == 2 && g0 && g0->dims.size() == 2,
             SPECDEC_EFORMAT, "sme: embed_tokens, layers.0.k_proj and layers.0.gate_proj are required");
    specdec_model_config c{};
    c.hidden = (int)num("hidden_dim", emb->dims[1]);
    c.layers = (int)num("num_layers", 0);
    c.n_q_heads = (int)num("num_heads", 0);
    SD_CHECK(c.hidden > 0 && c.layers > 0 && c.n_q_heads > 0, SPECDEC_EFORMAT,
             "sme: config needs num_layers and num_heads");
    c.head_dim = (int)num("head_dim", c.hidden / c.n_q_heads);
    SD_CHECK(c.head_dim > 0, SPECDEC_EFORMAT, "sme: bad head_dim");
    c.n_kv_heads = (int)num("num_kv_heads", num("num_key_value_heads", (double)(k0->dims[0] / (uint32_t)c.head_dim)));
    c.ffn = (int)g0->dims[0];
    c.vocab = (int)num("vocab_size", emb->dims[0]);
    int heads = 0;
    while (sme_role(f, "mtp", heads)) ++heads;
    c.n_mtp_heads = heads ? heads : (int)num("num_mtp_heads", 3);
    c.block_size = 16;
    c.rms_eps = (float)num("rms_norm_eps", 1e-5);
    c.rope_theta = (float)num("rope_theta", 10000.0);
    *mc = c;
    return SPECDEC_OK;
}

extern "C" int specdec_w4_convert(const void* src, int src_f32, const float* row_scales, const float* fold, int rows,
                                  int K, void* tiled, int N, int row0, int layout, void* stream) {
    SD_CHECK(src && tiled && rows >= 0 && K > 0 && K % 8 == 0 && layout >= 0 && layout <= 2, SPECDEC_EINVAL,
             "w4_convert: bad argument");
    SD_CHECK(src_f32 || row_scales, SPECDEC_EINVAL, "w4_convert: int8 rows need row scales");
    if (layout == 0) {
        SD_CHECK(row0 >= 0 && (int64_t)row0 + rows <= N, SPECDEC_EINVAL, "w4_convert: rows past N");
    } else {
        SD_CHECK(row0 == 0 && 128 * 2 * (((int64_t)rows + 127) / 128) <= (((int64_t)N + 255) / 256) * 256,
                 SPECDEC_EINVAL, "w4_convert: gate/up rows past N");
    }
    W4Source s{};
    s.K = K;
    s.fold = fold;
    if (src_f32) {
        s.f32 = static_cast<const float*>(src);
    } else {
        s.q8 = static_cast<const int8_t*>(src);
        s.rs = row_scales;
    }
    return w4_convert_launch(s, rows, row0, layout, static_cast<uint8_t*>(tiled), (K + 127) / 128, as_stream(stream));
}
