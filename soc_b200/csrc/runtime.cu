// Host runtime and C ABI of soc_b200: bundle loading into HBM, the paged KV
// cache, and the prefill / decode / generate drivers.
//
// The host side mirrors the reference runtime's objects (SongWooYoung/SoC):
//   soc_model  <-> QwenModelLoader::LoadModel -> QwenCausalLM   (Mac/cpu/src/qwen_model_loader.cpp:35-93)
//   soc_kv     <-> TensorKVCache / Metal KVCache                 (Mac/cpu/src/kv_cache.cpp, Mac/gpu/src/runtime/kv_cache.mm)
//   prefill / decode / generate <-> GenerationContext            (Mac/gpu/src/runtime/generation_context.cpp)
#include <sys/stat.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/soc_b200.h"
#include "common.cuh"
#include "decode_mk.h"
#include "gemm_tc.h"
#include "nccl_rt.h"
#include "tp_allreduce.h"
#include "json.hpp"
#include "kernels.h"

using namespace socb;

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
}  // namespace

void socb::set_last_error(const std::string& message) { g_last_error = message; }

namespace {

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return SOC_B200_OK;
    } catch (const Error& e) {
        return fail(e.code, e.what());
    } catch (const std::exception& e) {
        return fail(SOC_B200_ERR_INVALID, e.what());
    }
}

[[noreturn]] void throw_fmt(const std::string& m) { throw Error(SOC_B200_ERR_FORMAT, m); }

// ------------------------------------------------------------------ manifest
struct TensorRecord {
    std::string name, file, dtype;
    std::vector<size_t> shape;
    size_t byte_size = 0;
};

struct Config {
    size_t hidden = 0, inter = 0, layers = 0, hq = 0, hkv = 0, hd = 0, vocab = 0, max_pos = 40960;
    double eps = 0, theta = 0;
    bool tied = true;
};

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error(SOC_B200_ERR_IO, "failed to open file: " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

std::string dir_of(const std::string& p) {
    const auto pos = p.find_last_of('/');
    return pos == std::string::npos ? std::string(".") : p.substr(0, pos);
}

size_t dtype_width(const std::string& d) {
    if (d == "float32" || d == "int32") return 4;
    if (d == "float16" || d == "bfloat16" || d == "uint16") return 2;
    if (d == "int64") return 8;
    if (d == "int8" || d == "uint8" || d == "bool") return 1;
    throw_fmt("unsupported dtype string: " + d);
}

struct Manifest {
    std::string dir;
    Json config;
    std::vector<TensorRecord> tensors;
    const TensorRecord& find(const std::string& n) const {
        for (auto& t : tensors)
            if (t.name == n) return t;
        throw_fmt("missing tensor in manifest: " + n);
    }
};

// ManifestLoader::LoadFromFile + StartupValidator::ValidateManifest
// (Mac/cpu/src/runtime_assets.cpp:138-168, startup_validator.cpp:5-23).
Manifest load_manifest(const std::string& path) {
    Json root;
    try {
        root = JsonReader(read_file(path)).parse();
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw_fmt(e.what());
    }
    Manifest m;
    m.dir = dir_of(path);
    try {
        if (root.at("format").as_string() != "soc.cpp.llm_export") throw_fmt("manifest format must be soc.cpp.llm_export");
        if (root.at("format_version").as_int64() < 2) throw_fmt("manifest format_version must be at least 2");
        root.at("export_dtype").as_string();
        if (!root.contains("config") || !root.at("config").is_object()) throw_fmt("manifest config must be a JSON object");
        m.config = root.at("config");
        for (const Json& t : root.at("tensors").as_array()) {
            TensorRecord r;
            r.name = t.at("name").as_string();
            r.file = m.dir + "/" + t.at("file").as_string();
            r.dtype = t.at("dtype").as_string();
            for (const Json& s : t.at("shape").as_array()) r.shape.push_back(static_cast<size_t>(s.as_int64()));
            r.byte_size = static_cast<size_t>(t.at("byte_size").as_int64());
            t.at("source_shard").as_string();
            m.tensors.push_back(std::move(r));
        }
        if (m.tensors.empty()) throw_fmt("manifest must contain at least one tensor");
        if (!root.contains("tokenizer_runtime_file") || root.at("tokenizer_runtime_file").as_string().empty())
            throw_fmt("manifest must reference tokenizer_runtime_file");
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw_fmt(e.what());
    }
    return m;
}

// Qwen3Config::FromJson + Validate (Mac/cpu/src/qwen3_config.cpp:20-66).
Config read_config(const Json& c) {
    Config k;
    try {
        if (c.at("model_type").as_string() != "qwen3") throw_fmt("config model_type must be qwen3");
        k.hidden = static_cast<size_t>(c.at("hidden_size").as_int64());
        k.inter = static_cast<size_t>(c.at("intermediate_size").as_int64());
        k.layers = static_cast<size_t>(c.at("num_hidden_layers").as_int64());
        k.hq = static_cast<size_t>(c.at("num_attention_heads").as_int64());
        k.hkv = static_cast<size_t>(c.at("num_key_value_heads").as_int64());
        k.hd = static_cast<size_t>(c.at("head_dim").as_int64());
        k.eps = c.at("rms_norm_eps").as_number();
        k.theta = c.at("rope_theta").as_number();
        k.tied = c.at("tie_word_embeddings").as_bool();
        if (c.at("torch_dtype").as_string().empty()) throw_fmt("torch_dtype must not be empty");
        k.vocab = static_cast<size_t>(c.at("vocab_size").as_int64());
        if (c.contains("max_position_embeddings")) k.max_pos = static_cast<size_t>(c.at("max_position_embeddings").as_int64());
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw_fmt(e.what());
    }
    if (k.hidden == 0 || k.inter == 0 || k.layers == 0) throw_fmt("qwen3 config dimensions must be non-zero");
    if (k.hq == 0 || k.hkv == 0 || k.hd == 0) throw_fmt("qwen3 attention dimensions must be non-zero");
    if (k.hidden % k.hq != 0) throw_fmt("hidden_size must be divisible by num_attention_heads");
    if (k.hq % k.hkv != 0) throw_fmt("num_attention_heads must be divisible by num_key_value_heads");
    if (k.eps <= 0.0 || k.theta <= 0.0) throw_fmt("qwen3 normalization and rope parameters must be positive");
    if (k.vocab == 0) throw_fmt("vocab_size must be non-zero");
    // Limits of this implementation's kernels.
    if (k.hd != 64 && k.hd != 128) throw_fmt("soc_b200 supports head_dim 64 or 128");
    if (k.hq / k.hkv > 8) throw_fmt("soc_b200 supports at most 8 query heads per kv head");
    if (k.hidden % 256 != 0 || k.inter % 256 != 0 || (k.hq * k.hd) % 256 != 0)
        throw_fmt("soc_b200 needs hidden, intermediate and q width to be multiples of 256");
    if (k.max_pos == 0 || k.max_pos > (1u << 20)) k.max_pos = 40960;
    return k;
}

// WeightLoader::LoadTensor checks (Mac/cpu/src/weight_loader.cpp:17-30), then reads the bytes.
// The record's own consistency first, then the file, then the shape the model expects (the
// order in which WeightLoader::LoadTensor and RequireFloatingWeight report them).
std::vector<char> load_record(const TensorRecord& r, const std::vector<size_t>& expect_shape) {
    size_t numel = 1;
    for (size_t s : r.shape) numel *= s;
    const size_t expect = numel * dtype_width(r.dtype);
    if (expect != r.byte_size) throw_fmt("tensor record byte_size does not match dtype and shape for: " + r.name);
    struct stat st {};
    if (stat(r.file.c_str(), &st) != 0) throw Error(SOC_B200_ERR_IO, "failed to open tensor file: " + r.file);
    if (static_cast<size_t>(st.st_size) < r.byte_size)
        throw Error(SOC_B200_ERR_IO, "tensor file is smaller than expected byte_size for: " + r.name);
    if (r.shape != expect_shape) throw_fmt("model loader encountered unexpected shape for: " + r.name);
    std::vector<char> buf(r.byte_size);
    FILE* f = std::fopen(r.file.c_str(), "rb");
    if (!f) throw Error(SOC_B200_ERR_IO, "failed to open tensor file: " + r.file);
    const size_t got = std::fread(buf.data(), 1, r.byte_size, f);
    std::fclose(f);
    if (got != r.byte_size) throw Error(SOC_B200_ERR_IO, "short read for tensor: " + r.name);
    return buf;
}

float half_bits_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ee = -14;
            while (!(m & 0x400)) {
                m <<= 1;
                --ee;
            }
            bits = sign | (static_cast<uint32_t>(ee + 127) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 0x1f) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Norm weights are kept in fp32 on the device (exact for fp16 / bf16 sources).
std::vector<float> to_f32(const TensorRecord& r, const std::vector<char>& b) {
    size_t n = b.size() / dtype_width(r.dtype);
    std::vector<float> out(n);
    if (r.dtype == "float32") {
        std::memcpy(out.data(), b.data(), n * 4);
    } else if (r.dtype == "float16") {
        const uint16_t* p = reinterpret_cast<const uint16_t*>(b.data());
        for (size_t i = 0; i < n; ++i) out[i] = half_bits_to_float(p[i]);
    } else if (r.dtype == "bfloat16") {
        const uint16_t* p = reinterpret_cast<const uint16_t*>(b.data());
        for (size_t i = 0; i < n; ++i) {
            uint32_t bits = static_cast<uint32_t>(p[i]) << 16;
            std::memcpy(&out[i], &bits, 4);
        }
    } else {
        throw_fmt("model loader requires floating-point weights for: " + r.name);
    }
    return out;
}

uint16_t float_to_half_bits(float f) {
    const __half h = __float2half_rn(f);
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
}


// ------------------------------------------------- linear matrices in the device format
// Group-wise quantised records (bundle extension): dtype "int8_g64" ([out, in] int8) or
// "int4_g32" ([out, in/2] bytes, two's complement nibbles, low nibble = even column), each
// with a "<name>.scales" float16 record [out, in/group].  Value = float(q) * float(scale).
int quant_group(int fmt) { return fmt == WF_I8G64 ? 64 : fmt == WF_I4G32 ? 32 : 0; }
size_t fmt_row_bytes(int fmt, size_t cols) {
    return fmt == WF_I8G64 ? cols : fmt == WF_I4G32 ? cols / 2 : cols * 2;
}
int fmt_of_dtype(const std::string& d) {
    if (d == "int8_g64") return WF_I8G64;
    if (d == "int4_g32") return WF_I4G32;
    if (d == "bfloat16") return WF_BF16;
    if (d == "float16" || d == "float32") return WF_F16;
    return 0;
}

struct HostMat {
    std::vector<uint8_t> data;     // rows * fmt_row_bytes
    std::vector<uint16_t> scales;  // rows * cols / group fp16 bits (quantised formats)
};

// Symmetric group quantisation, the per-group extension of QuantizeMatMulRhs8
// (Mac/cpu/header/matrix_ops.h:42-73): s = fp16(max|w| / qmax), q = clamp(rint(w / s)).
void quantize_rows(const float* w, size_t rows, size_t cols, int fmt, HostMat& out) {
    const int g = quant_group(fmt);
    const float qmax = fmt == WF_I8G64 ? 127.0f : 7.0f;
    const size_t ng = cols / g;
    out.data.assign(rows * fmt_row_bytes(fmt, cols), 0);
    out.scales.assign(rows * ng, 0);
    std::vector<int8_t> q(g);
    for (size_t r = 0; r < rows; ++r) {
        for (size_t gi = 0; gi < ng; ++gi) {
            const float* wg = w + r * cols + gi * g;
            float amax = 0.0f;
            for (int i = 0; i < g; ++i) amax = std::max(amax, std::fabs(wg[i]));
            const uint16_t sb = float_to_half_bits(amax / qmax);
            const float s = half_bits_to_float(sb);
            for (int i = 0; i < g; ++i) {
                float v = s == 0.0f ? 0.0f : std::nearbyint(wg[i] / s);
                v = std::min(qmax, std::max(-qmax, v));
                q[i] = static_cast<int8_t>(v);
            }
            out.scales[r * ng + gi] = sb;
            uint8_t* dst = out.data.data() + r * fmt_row_bytes(fmt, cols) + fmt_row_bytes(fmt, gi * g);
            if (fmt == WF_I8G64) {
                std::memcpy(dst, q.data(), g);
            } else {
                for (int i = 0; i < g; i += 2)
                    dst[i / 2] = static_cast<uint8_t>((q[i] & 0xF) | ((q[i + 1] & 0xF) << 4));
            }
        }
    }
}

std::vector<float> dequantize_rows(const std::vector<char>& b, const std::vector<char>& sb, size_t rows, size_t cols,
                                   int fmt) {
    const int g = quant_group(fmt);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(sb.data());
    const uint8_t* d = reinterpret_cast<const uint8_t*>(b.data());
    std::vector<float> out(rows * cols);
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) {
            int q;
            if (fmt == WF_I8G64) {
                q = static_cast<int8_t>(d[r * cols + c]);
            } else {
                const uint8_t byte = d[r * (cols / 2) + c / 2];
                q = (c & 1) ? (byte >> 4) : (byte & 0xF);
                if (q > 7) q -= 16;
            }
            out[r * cols + c] = static_cast<float>(q) * half_bits_to_float(sc[r * (cols / g) + c / g]);
        }
    return out;
}

// Sub-block [r0, r0 + nr) x [c0, c0 + nc) of a row-major matrix (tensor-parallel shard).
struct Block {
    size_t r0 = 0, nr = 0, c0 = 0, nc = 0;
};

// Row-major bytes of `blk` from a matrix whose rows hold `cols` elements of `row_bytes(cols)`.
template <typename RB>
std::vector<char> cut(const std::vector<char>& b, size_t cols, const Block& blk, RB row_bytes) {
    const size_t rb = row_bytes(cols), ob = row_bytes(blk.nc), off = row_bytes(blk.c0);
    std::vector<char> o(blk.nr * ob);
    for (size_t r = 0; r < blk.nr; ++r) std::memcpy(o.data() + r * ob, b.data() + (blk.r0 + r) * rb + off, ob);
    return o;
}

// Reads linear `name` ([rows, cols]), keeps the block `blk` (default: all of it) and
// returns it in device format `fmt`.
HostMat prepare_matrix(const Manifest& man, const std::string& name, size_t rows, size_t cols, int fmt,
                       Block blk = Block{}) {
    const TensorRecord& r = man.find(name);
    if (blk.nr == 0) blk = Block{0, rows, 0, cols};
    if (blk.r0 + blk.nr > rows || blk.c0 + blk.nc > cols) throw Error(SOC_B200_ERR_INVALID, "shard outside " + name);
    HostMat out;
    const int src = fmt_of_dtype(r.dtype);
    std::vector<float> f32;
    const size_t nr = blk.nr, nc = blk.nc;
    if (src == WF_I8G64 || src == WF_I4G32) {
        if (r.shape != std::vector<size_t>{rows, cols})
            throw_fmt("model loader encountered unexpected shape for: " + name);
        const int g = quant_group(src);
        if (cols % g != 0) throw_fmt("quantised tensor columns are not a multiple of the group for: " + name);
        if (blk.c0 % g != 0 || nc % g != 0) throw Error(SOC_B200_ERR_INVALID, "shard splits a quantisation group: " + name);
        TensorRecord raw = r;
        raw.dtype = "uint8";
        raw.shape = {rows * fmt_row_bytes(src, cols)};
        const std::vector<char> b = cut(load_record(raw, raw.shape), cols, blk,
                                        [&](size_t c) { return fmt_row_bytes(src, c); });
        const TensorRecord& rs = man.find(name + ".scales");
        if (rs.dtype != "float16") throw_fmt("quantisation scales must be float16 for: " + name);
        const std::vector<char> sb = cut(load_record(rs, {rows, cols / g}), cols, blk,
                                         [&](size_t c) { return c / g * 2; });
        if (src == fmt) {
            out.data.assign(b.begin(), b.end());
            out.scales.resize(nr * (nc / g));
            std::memcpy(out.scales.data(), sb.data(), sb.size());
            return out;
        }
        f32 = dequantize_rows(b, sb, nr, nc, src);
    } else {
        const size_t w = dtype_width(r.dtype);
        std::vector<char> b = load_record(r, {rows, cols});
        if (nr != rows || nc != cols) b = cut(b, cols, blk, [&](size_t c) { return c * w; });
        const bool same = (fmt == WF_F16 && r.dtype == "float16") || (fmt == WF_BF16 && r.dtype == "bfloat16");
        if (same) {
            out.data.assign(b.begin(), b.end());
            return out;
        }
        f32 = to_f32(r, b);
    }
    if (fmt == WF_I8G64 || fmt == WF_I4G32) {
        if (nc % quant_group(fmt) != 0) throw_fmt("in_features is not a multiple of the quantisation group: " + name);
        quantize_rows(f32.data(), nr, nc, fmt, out);
        return out;
    }
    out.data.resize(nr * nc * 2);
    uint16_t* d = reinterpret_cast<uint16_t*>(out.data.data());
    for (size_t i = 0; i < f32.size(); ++i) {
        if (fmt == WF_F16) {
            d[i] = float_to_half_bits(f32[i]);
        } else {
            const __nv_bfloat16 bb = __float2bfloat16_rn(f32[i]);
            std::memcpy(&d[i], &bb, 2);
        }
    }
    return out;
}

// WeightLoader::LoadTensor's record checks (weight_loader.cpp:17-30) without reading the data:
// byte_size against the record's dtype and shape, then the file's length.
void check_record(const TensorRecord& r) {
    size_t numel = 1;
    for (size_t s : r.shape) numel *= s;
    if (numel * dtype_width(r.dtype) != r.byte_size)
        throw_fmt("tensor record byte_size does not match dtype and shape for: " + r.name);
    struct stat st {};
    if (stat(r.file.c_str(), &st) != 0) throw Error(SOC_B200_ERR_IO, "failed to open tensor file: " + r.file);
    if (static_cast<size_t>(st.st_size) < r.byte_size)
        throw Error(SOC_B200_ERR_IO, "tensor file is smaller than expected byte_size for: " + r.name);
}

// RequireFloatingWeight (qwen_model_loader.cpp:17-26): the record, a float type, the expected
// shape.  Block linears may also be group-quantised records with their scales (this library's
// bundle extension).
void check_weight(const Manifest& man, const std::string& name, const std::vector<size_t>& shape,
                  bool may_be_quantised = false) {
    const TensorRecord& r = man.find(name);
    const int src = fmt_of_dtype(r.dtype);
    if (may_be_quantised && (src == WF_I8G64 || src == WF_I4G32)) {
        const size_t rows = shape[0], cols = shape[1];
        if (r.shape != shape) throw_fmt("model loader encountered unexpected shape for: " + name);
        const int g = quant_group(src);
        if (cols % g != 0) throw_fmt("quantised tensor columns are not a multiple of the group for: " + name);
        TensorRecord raw = r;
        raw.dtype = "uint8";
        raw.shape = {rows * fmt_row_bytes(src, cols)};
        check_record(raw);
        const TensorRecord& rs = man.find(name + ".scales");
        if (rs.dtype != "float16") throw_fmt("quantisation scales must be float16 for: " + name);
        check_record(rs);
        if (rs.shape != std::vector<size_t>{rows, cols / g})
            throw_fmt("model loader encountered unexpected shape for: " + rs.name);
        return;
    }
    check_record(r);
    if (r.dtype != "float16" && r.dtype != "bfloat16" && r.dtype != "float32")
        throw_fmt("model loader requires floating-point weights for: " + name);
    if (r.shape != shape) throw_fmt("model loader encountered unexpected shape for: " + name);
}

// RuntimePipeline::LoadBundle's checks (Mac/cpu/src/runtime_pipeline.cpp:36-41) on the host:
// ManifestLoader + TokenizerRuntimeLoader, StartupValidator::ValidateManifestAndTokenizer, and
// every record QwenModelLoader::LoadModel reads (qwen_model_loader.cpp:35-93), in that order.
// Weights are not read; their files are only measured.
void validate_bundle(const std::string& manifest_path) {
    const Manifest man = load_manifest(manifest_path);
    std::string tok_path;
    {
        size_t n = 0;
        soc_b200_manifest_tokenizer_path(manifest_path.c_str(), nullptr, 0, &n);
        tok_path.assign(n + 1, '\0');
        if (soc_b200_manifest_tokenizer_path(manifest_path.c_str(), &tok_path[0], tok_path.size(), &n) != SOC_B200_OK)
            throw Error(SOC_B200_ERR_FORMAT, soc_b200_last_error());
        tok_path.resize(n);
    }
    soc_tokenizer* tok = nullptr;
    int rc = soc_b200_tokenizer_load(tok_path.c_str(), &tok);
    if (rc != SOC_B200_OK) throw Error(rc, soc_b200_last_error());
    const Config c = read_config(man.config);
    rc = soc_b200_tokenizer_check_model(tok, static_cast<long long>(c.vocab));
    soc_b200_tokenizer_free(tok);
    if (rc != SOC_B200_OK) throw Error(rc, soc_b200_last_error());

    const size_t H = c.hidden, I = c.inter, D = c.hd, QW = c.hq * D, KW = c.hkv * D;
    check_weight(man, "model.embed_tokens.weight", {c.vocab, H});
    for (size_t l = 0; l < c.layers; ++l) {  // the reference loader's order
        const std::string p = "model.layers." + std::to_string(l) + ".";
        check_weight(man, p + "input_layernorm.weight", {H});
        check_weight(man, p + "self_attn.q_proj.weight", {QW, H}, true);
        check_weight(man, p + "self_attn.k_proj.weight", {KW, H}, true);
        check_weight(man, p + "self_attn.v_proj.weight", {KW, H}, true);
        check_weight(man, p + "self_attn.o_proj.weight", {H, QW}, true);
        check_weight(man, p + "self_attn.q_norm.weight", {D});
        check_weight(man, p + "self_attn.k_norm.weight", {D});
        check_weight(man, p + "post_attention_layernorm.weight", {H});
        check_weight(man, p + "mlp.gate_proj.weight", {I, H}, true);
        check_weight(man, p + "mlp.up_proj.weight", {I, H}, true);
        check_weight(man, p + "mlp.down_proj.weight", {H, I}, true);
    }
    check_weight(man, "model.norm.weight", {H});
    if (!c.tied) check_weight(man, "lm_head.weight", {c.vocab, H});
}

}  // namespace

// ------------------------------------------------------------------- objects
struct soc_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int sm_count = 0;
    int* d_err = nullptr;
    void* lin_scratch = nullptr;  // soc_b200_linear tensor-core path: input rows (hi, lo) + fp16 weights
    size_t lin_scratch_bytes = 0;
    float* gemm_ws = nullptr;     // split-K partial tiles of the tensor-core GEMM (TC_WS_FLOATS)
    float* ws() {
        if (!gemm_ws) SOCB_CUDA(cudaMalloc(&gemm_ws, TC_WS_FLOATS * sizeof(float)));
        return gemm_ws;
    }
};

struct LayerW {
    void* wqkv = nullptr;  // [(hq + 2 hkv) * hd, hidden]  q rows, then k, then v
    void* wo = nullptr;    // [hidden, hq * hd]
    void* wgu = nullptr;   // [2 * inter, hidden] rows (2j, 2j+1) = (gate_j, up_j)
    void* wd = nullptr;    // [hidden, inter]
    // fp16 group scales [rows, in / group] of the same matrices (quantised formats only)
    void *sqkv = nullptr, *so = nullptr, *sgu = nullptr, *sd = nullptr;
    // TMA descriptors of the four matrices for the tensor-core GEMM (fp16 / bf16 only)
    CUtensorMap tm_qkv{}, tm_o{}, tm_gu{}, tm_d{};
    float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

struct soc_model {
    soc_ctx* ctx = nullptr;
    Config cfg;       // this rank's shard: q/kv heads and intermediate divided by tp_size
    Config cfg_full;  // the whole model
    // tensor parallelism (Megatron-style): column-parallel q/k/v and gate/up, row-parallel
    // o_proj and down_proj followed by an all-reduce of the residual stream, vocab-parallel
    // lm_head with a merged argmax
    int tp_rank = 0, tp_size = 1;
    ncclComm_t comm = nullptr;
    TpExchange* ar = nullptr;  // peer-memory all-reduce (opt-in), else NCCL
    int v_loc = 0, v_off = 0;                 // lm_head rows held here
    float* logits_all = nullptr;              // [tp][rows][v_loc] gathered logits
    int logits_all_rows = 0;
    unsigned long long* d_keys = nullptr;     // [tp][rows] argmax keys (this rank's at tp_rank)
    int wfmt = WF_F16;  // block linears
    int efmt = WF_F16;  // embedding / lm_head
    void* embed = nullptr;
    void* lm_head = nullptr;  // == embed when tied
    float* final_norm = nullptr;
    std::vector<LayerW> layers;
    float2* rope_cs = nullptr;
    int rope_len = 0;
    std::vector<void*> allocs;
    // workspace (grown on demand)
    int ws_rows = 0;
    float *h = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *act = nullptr;
    int *d_tokens = nullptr, *d_seq = nullptr, *d_pos = nullptr, *d_next = nullptr;
    // tensor-core GEMM path (gemm_tc.cu)
    bool tc_ok = false;
    int gfmt = WF_F16;                         // GEMM element type (fp16 for fp16 and quantised models)
    void *xa = nullptr, *xa_lo = nullptr;      // [ws_rows, max(hidden, q width)] GEMM input rows (hi, lo)
    void *acth = nullptr, *acth_lo = nullptr;  // [ws_rows, inter] SwiGLU output = down_proj input (hi, lo)
    void* wdq = nullptr;                       // fp16 expansion of one quantised matrix (quantised models)
    CUtensorMap tm_lm{};                       // descriptor of the lm_head rows held here
    CUtensorMap tm_dq_qkv{}, tm_dq_o{}, tm_dq_gu{}, tm_dq_d{};  // descriptors over wdq, one per shape
    float* logits = nullptr;
    int logits_rows = 0;
    int logits_last_rows = 0;  // rows of m->logits the last prefill / decode left (0: none)
    unsigned long long* topk_cand = nullptr;  // top-k scratch: candidates, then k logits and k ids
    float* topk_vals = nullptr;
    int* topk_ids = nullptr;
    float* attn_scratch = nullptr;
    size_t attn_scratch_floats = 0;
    // device-fed decode loop (CUDA graph of one step, replayed per token)
    struct LoopState {
        int* out;
        int seq, start, step;
        int steps, eos;  // the device loop runs while step < steps and out[step] != eos (eos >= 0)
    };
    LoopState* d_loop = nullptr;
    cudaGraphExec_t step_graph = nullptr;  // the decode loop: a WHILE node around one step
    int loop_steps_queued = 0;             // steps the last graph decode loop was launched for
    // short prefill chunks replayed as one CUDA graph (the launches, not the bytes, bound them)
    struct PrefillKey {
        const void *kv, *h, *xa, *logits;
        unsigned long long epoch;  // buf_epoch at capture
        int seq, start, n, lm;
        float temperature;
        bool operator==(const PrefillKey& o) const {
            return kv == o.kv && h == o.h && xa == o.xa && logits == o.logits && epoch == o.epoch && seq == o.seq &&
                   start == o.start && n == o.n && lm == o.lm && temperature == o.temperature;
        }
    };
    cudaGraphExec_t pf_graph = nullptr;
    PrefillKey pf_key{};
    long long pf_graph_kernels = 0;
    bool pf_graph_broken = false;  // a capture failed once: prefill chunks run directly
    const soc_kv* graph_kv = nullptr;
    int graph_splits = 0;
    unsigned long long graph_epoch = 0;  // buf_epoch when step_graph was captured
    long long graph_kernels = 0;
    // persistent batch-1 decode kernel (decode_mk.cu)
    bool mk_ok = false;
    // Sampler(SamplerConfig) of the reference (Mac/cpu/header/sampler.h:9-12): picks maximise
    // logit / temperature; top_k only validated (the best of the top k is the maximum).
    float temperature = 1.0f;
    size_t top_k = 1;
    int mk_grid = 0;
    MKLayer* d_mk_layers = nullptr;
    void* mk_lm_tiles = nullptr;              // the lm_head in the kernel's tiled layout
    unsigned long long* mk_best = nullptr;
    int mk_best_n = 0;
    unsigned long long* mk_part = nullptr;    // split-K attention partials (tagged words)
    size_t mk_part_n = 0;
    int* mk_ids = nullptr;
    unsigned long long* mk_vec = nullptr;     // h | qkv | attn | act as tagged words
    size_t mk_vec_n = 0;
    unsigned mk_tag = 0;                      // tags used so far on mk_vec / mk_part

    void* dmalloc(size_t bytes) {
        void* p = nullptr;
        SOCB_CUDA(cudaMalloc(&p, bytes));
        allocs.push_back(p);
        return p;
    }
    // Bumped whenever a buffer is freed: a captured graph that baked in the old pointer is stale.
    unsigned long long buf_epoch = 0;
    void dfree(void* p, bool graphs_may_hold = true) {
        if (!p) return;
        if (graphs_may_hold) ++buf_epoch;
        cudaFree(p);
        for (auto& a : allocs)
            if (a == p) a = nullptr;
    }
    size_t qkv_dim() const { return (cfg.hq + 2 * cfg.hkv) * cfg.hd; }
};

struct soc_kv {
    soc_model* m = nullptr;
    int max_seqs = 0, page_tokens = 16, num_pages = 0, max_pages = 0;
    __half* k = nullptr;  // [layers][num_pages][hkv][page_tokens][hd]
    __half* v = nullptr;
    int* d_page_table = nullptr;  // [max_seqs][max_pages]
    std::vector<int> lengths;
    std::vector<std::vector<int>> pages;
    std::vector<int> free_pages;
    size_t layer_stride() const { return static_cast<size_t>(num_pages) * m->cfg.hkv * page_tokens * m->cfg.hd; }
    CUtensorMap tmk{}, tmv{};  // TMA views of the pools for the page-streaming attention
    bool tm_ok = false;
    KVLayerView view(int layer) const {
        KVLayerView v_{k + layer * layer_stride(), v + layer * layer_stride(), d_page_table, max_pages, page_tokens};
        if (tm_ok) {
            v_.tmk = &tmk;
            v_.tmv = &tmv;
            v_.row0 = static_cast<int>(static_cast<size_t>(layer) * num_pages * m->cfg.hkv * page_tokens);
        }
        return v_;
    }
    void check_seq(int seq) const {
        if (seq < 0 || seq >= max_seqs) throw Error(SOC_B200_ERR_INVALID, "kv cache sequence index out of range");
    }
    // Make room for positions [0, new_len) of `seq` (host page allocator + device page table).
    void reserve(int seq, int new_len, cudaStream_t st) {
        if (new_len > max_pages * page_tokens)
            throw Error(SOC_B200_ERR_CAPACITY, "GenerationContext sequence length would exceed max_sequence_length");
        const int need = (new_len + page_tokens - 1) / page_tokens;
        auto& pv = pages[seq];
        const int before = static_cast<int>(pv.size());
        if (need <= before) return;
        if (static_cast<int>(free_pages.size()) < need - before)
            throw Error(SOC_B200_ERR_CAPACITY, "kv cache out of pages");
        while (static_cast<int>(pv.size()) < need) {
            pv.push_back(free_pages.back());
            free_pages.pop_back();
        }
        SOCB_CUDA(cudaMemcpyAsync(d_page_table + static_cast<size_t>(seq) * max_pages + before, pv.data() + before,
                                  sizeof(int) * (need - before), cudaMemcpyHostToDevice, st));
    }
    void reset(int seq) {
        for (int p : pages[seq]) free_pages.push_back(p);
        pages[seq].clear();
        lengths[seq] = 0;
    }
};

namespace {

void ensure_workspace(soc_model* m, int rows) {
    if (rows <= m->ws_rows) return;
    const Config& c = m->cfg;
    int r = 16;
    while (r < rows) r *= 2;
    for (void* p : {static_cast<void*>(m->h), static_cast<void*>(m->qkv), static_cast<void*>(m->q),
                    static_cast<void*>(m->att), static_cast<void*>(m->act), static_cast<void*>(m->d_tokens),
                    static_cast<void*>(m->d_seq), static_cast<void*>(m->d_pos), static_cast<void*>(m->d_next)})
        m->dfree(p);
    m->h = static_cast<float*>(m->dmalloc(sizeof(float) * r * c.hidden));
    m->qkv = static_cast<float*>(m->dmalloc(sizeof(float) * r * m->qkv_dim()));
    m->q = static_cast<float*>(m->dmalloc(sizeof(float) * r * c.hq * c.hd));
    m->att = static_cast<float*>(m->dmalloc(sizeof(float) * r * c.hq * c.hd));
    m->act = static_cast<float*>(m->dmalloc(sizeof(float) * r * c.inter));
    m->d_tokens = static_cast<int*>(m->dmalloc(sizeof(int) * r));
    m->d_seq = static_cast<int*>(m->dmalloc(sizeof(int) * r));
    m->d_pos = static_cast<int*>(m->dmalloc(sizeof(int) * r));
    m->d_next = static_cast<int*>(m->dmalloc(sizeof(int) * r));
    if (m->tc_ok) {
        for (void* p : {m->xa, m->xa_lo, m->acth, m->acth_lo}) m->dfree(p);
        m->xa = m->dmalloc(2 * static_cast<size_t>(r) * std::max(c.hidden, c.hq * c.hd));
        m->xa_lo = m->dmalloc(2 * static_cast<size_t>(r) * std::max(c.hidden, c.hq * c.hd));
        m->acth = m->dmalloc(2 * static_cast<size_t>(r) * c.inter);
        m->acth_lo = m->dmalloc(2 * static_cast<size_t>(r) * c.inter);
    }
    m->ws_rows = r;
}

void ensure_logits(soc_model* m, int rows) {
    if (rows <= m->logits_rows) return;
    m->dfree(m->logits);
    m->logits = static_cast<float*>(m->dmalloc(sizeof(float) * rows * m->v_loc));
    m->logits_rows = rows;
    m->dfree(m->d_keys);
    m->d_keys = static_cast<unsigned long long*>(m->dmalloc(sizeof(unsigned long long) * rows * m->tp_size));
}

void ensure_attn_scratch(soc_model* m, size_t floats) {
    if (floats <= m->attn_scratch_floats) return;
    m->dfree(m->attn_scratch);
    m->attn_scratch = static_cast<float*>(m->dmalloc(sizeof(float) * floats));
    m->attn_scratch_floats = floats;
}

void check_device_error(soc_model* m) {
    int e = 0;
    SOCB_CUDA(cudaMemcpyAsync(&e, m->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, m->ctx->stream));
    SOCB_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (e != 0) {
        SOCB_CUDA(cudaMemsetAsync(m->ctx->d_err, 0, sizeof(int), m->ctx->stream));
        // a bounded wait gave up: if the peer exchange ran, its epochs may now disagree
        if ((e & DERR_WAIT_TIMEOUT) && m->ar != nullptr) m->ar->poisoned = true;
        if (e & DERR_TOKEN_RANGE) throw Error(SOC_B200_ERR_RANGE, "embedding input token id out of range");
        if (e & DERR_KV_RANGE) throw Error(SOC_B200_ERR_CAPACITY, "kv cache write position out of range");
        throw Error(SOC_B200_ERR_DEVICE, "device kernel reported error status " + std::to_string(e));
    }
}

// Run rows [0, n) (tokens/seq/pos already in m->d_tokens/d_seq/d_pos) through all layers.
// Afterwards m->h holds the residual stream; when lm_rows > 0 the logits of rows
// [lm_first, lm_first + lm_rows) go to m->logits and their greedy ids to m->d_next.
// Rows from which a prefill chunk's attention runs on the tensor-core flash kernel
// (default 32; SOC_B200_FLASH_MIN_ROWS overrides it, 0 disables it).
int flash_min_rows() {
    const char* e = std::getenv("SOC_B200_FLASH_MIN_ROWS");
    return e && *e ? std::atoi(e) : 32;
}

// The flash step of a prefill chunk runs on the tcgen05 kernel (attn_prefill_tc.cu: S and O in
// tensor memory); SOC_B200_PREFILL_ATTENTION=mma selects the mma.sync kernel (attn_prefill.cu).
bool prefill_attention_tc() {
    const char* e = std::getenv("SOC_B200_PREFILL_ATTENTION");
    return !(e && std::string(e) == "mma");
}

// pf_seq >= 0: the rows are positions pf_start .. pf_start + n - 1 of sequence pf_seq (a
// prefill chunk), which lets the attention use the flash kernel.
void forward_rows(soc_model* m, soc_kv* kv, int n, int max_visible, int lm_first, int lm_rows, int splits,
                  int pf_seq = -1, int pf_start = 0) {
    const Config& c = m->cfg;
    cudaStream_t st = m->ctx->stream;
    const float eps = static_cast<float>(c.eps);
    const int H = static_cast<int>(c.hidden), I = static_cast<int>(c.inter);
    const int QW = static_cast<int>(c.hq * c.hd), QKV = static_cast<int>(m->qkv_dim());
    Rows rows{m->d_tokens, m->d_seq, m->d_pos, n};
    if (m->ar != nullptr && m->ar->poisoned)
        throw Error(SOC_B200_ERR_DEVICE, "peer all-reduce: an earlier exchange timed out; reload the model");
    if (splits < 1) splits = attention_splits(n, static_cast<int>(c.hkv), max_visible);
    if (splits > 1) ensure_attn_scratch(m, static_cast<size_t>(n) * c.hq * splits * (c.hd + 2));
    launch_embed(m->efmt, m->embed, H, static_cast<int>(c.vocab), m->d_tokens, n, m->h, m->ctx->d_err, st);
    // Tensor-core GEMMs for the block linears once there are enough rows (group-quantised
    // weights are first expanded to fp16, one matrix at a time, into m->wdq).
    const bool quant = m->wfmt == WF_I8G64 || m->wfmt == WF_I4G32;
    const bool tc = m->tc_ok && tc_rows_ok(n, static_cast<long long>(2 * I), H, m->wfmt);
    const bool split = n <= tc_split_max_rows();
    const int gf = m->gfmt;
    CUtensorMap a_h{}, a_att{}, a_act{}, a_h_lo{}, a_att_lo{}, a_act_lo{};
    if (tc) {
        tc_make_map(&a_h, m->xa, gf, n, H, H, TC_BOX_A);
        tc_make_map(&a_att, m->xa, gf, n, QW, QW, TC_BOX_A);
        tc_make_map(&a_act, m->acth, gf, n, I, I, TC_BOX_A);
        if (split) {
            tc_make_map(&a_h_lo, m->xa_lo, gf, n, H, H, TC_BOX_A);
            tc_make_map(&a_att_lo, m->xa_lo, gf, n, QW, QW, TC_BOX_A);
            tc_make_map(&a_act_lo, m->acth_lo, gf, n, I, I, TC_BOX_A);
        }
    }
    void* xlo = split ? m->xa_lo : nullptr;
    float* gws = tc ? m->ctx->ws() : nullptr;
    // Weight operand of one linear: its own descriptor, or the fp16 expansion of a quantised matrix.
    auto wmap = [&](const CUtensorMap& own, const void* w, const void* sc, int rows_w, int cols_w,
                    const CUtensorMap& dq) -> const CUtensorMap& {
        if (!quant) return own;
        launch_dequant(m->wfmt, w, sc, rows_w, cols_w, WF_F16, m->wdq, st);
        return dq;
    };
    int* err = m->ctx->d_err;
    // Row-parallel o_proj / down_proj: rank 0 adds its partial product to the residual
    // stream, the other ranks store theirs, and the all-reduce sums them.
    const int res_mode = m->tp_rank == 0 ? LIN_RESIDUAL : LIN_STORE;
    auto tp_sum = [&] {
        if (m->tp_size <= 1) return;
        const size_t elems = static_cast<size_t>(n) * H;
        if (m->ar != nullptr && elems <= m->ar->max_elems && elems % 4 == 0)
            m->ar->all_reduce(m->h, elems, m->ctx->d_err, st);
        else
            nccl_check(nccl().all_reduce(m->h, m->h, elems, ncclFloat32, ncclSum, m->comm, st), "residual all-reduce");
    };
    const bool flash = pf_seq >= 0 && flash_min_rows() > 0 && n >= flash_min_rows();
    const bool flash_tc = flash && prefill_attention_tc() && kv->tm_ok;
    for (size_t l = 0; l < c.layers; ++l) {
        const LayerW& w = m->layers[l];
        if (tc) {
            launch_rows_to_half(gf, m->h, H, n, H, w.in_norm, eps, m->xa, xlo, H, st);
            launch_gemm_tc(gf, a_h, split ? &a_h_lo : nullptr, wmap(w.tm_qkv, w.wqkv, w.sqkv, QKV, H, m->tm_dq_qkv),
                           n, QKV, H, m->qkv, QKV, LIN_STORE, false, nullptr, gws, TC_WS_FLOATS, err, st);
        } else {
            launch_linear(m->wfmt, w.wqkv, w.sqkv, QKV, H, m->h, H, n, w.in_norm, eps, m->qkv, QKV, LIN_STORE, st);
        }
        launch_qk_norm_rope_kv(m->qkv, rows, static_cast<int>(c.hq), static_cast<int>(c.hkv), static_cast<int>(c.hd),
                               w.q_norm, w.k_norm, eps, m->rope_cs, m->rope_len, kv->view(static_cast<int>(l)), m->q,
                               m->ctx->d_err, st);
        if (flash && flash_tc)
            launch_flash_prefill_tc(m->q, n, static_cast<int>(c.hq), static_cast<int>(c.hkv), static_cast<int>(c.hd),
                                    pf_seq, pf_start, kv->view(static_cast<int>(l)), m->att, m->ctx->d_err, st);
        else if (flash)
            launch_flash_prefill(m->q, n, static_cast<int>(c.hq), static_cast<int>(c.hkv), static_cast<int>(c.hd),
                                 pf_seq, pf_start, kv->view(static_cast<int>(l)), m->att, st);
        else
            launch_attention(m->q, rows, splits, static_cast<int>(c.hq), static_cast<int>(c.hkv),
                             static_cast<int>(c.hd), kv->view(static_cast<int>(l)), m->att, m->attn_scratch,
                             m->attn_scratch_floats, m->ctx->d_err, st);
        if (tc) {
            launch_rows_to_half(gf, m->att, QW, n, QW, nullptr, eps, m->xa, xlo, QW, st);
            launch_gemm_tc(gf, a_att, split ? &a_att_lo : nullptr, wmap(w.tm_o, w.wo, w.so, H, QW, m->tm_dq_o), n, H,
                           QW, m->h, H, res_mode, false, nullptr, gws, TC_WS_FLOATS, err, st);
            tp_sum();
            launch_rows_to_half(gf, m->h, H, n, H, w.post_norm, eps, m->xa, xlo, H, st);
            launch_gemm_tc(gf, a_h, split ? &a_h_lo : nullptr, wmap(w.tm_gu, w.wgu, w.sgu, 2 * I, H, m->tm_dq_gu), n,
                           2 * I, H, m->acth, I, LIN_SWIGLU, true, split ? m->acth_lo : nullptr, gws, TC_WS_FLOATS,
                           err, st);
            launch_gemm_tc(gf, a_act, split ? &a_act_lo : nullptr, wmap(w.tm_d, w.wd, w.sd, H, I, m->tm_dq_d), n, H, I,
                           m->h, H, res_mode, false, nullptr, gws, TC_WS_FLOATS, err, st);
            tp_sum();
        } else {
            launch_linear(m->wfmt, w.wo, w.so, H, QW, m->att, QW, n, nullptr, eps, m->h, H, res_mode, st);
            tp_sum();
            launch_linear(m->wfmt, w.wgu, w.sgu, 2 * I, H, m->h, H, n, w.post_norm, eps, m->act, I, LIN_SWIGLU, st);
            launch_linear(m->wfmt, w.wd, w.sd, H, I, m->act, I, n, nullptr, eps, m->h, H, res_mode, st);
            tp_sum();
        }
    }
    if (lm_rows > 0) {
        ensure_logits(m, lm_rows);
        if (m->tc_ok && tc_rows_ok(lm_rows, m->v_loc, H, m->efmt)) {
            // many rows (batched decode): tensor-core GEMM over the vocab rows
            const bool lsplit = lm_rows <= tc_split_max_rows();
            CUtensorMap a_lm{}, a_lm_lo{};
            tc_make_map(&a_lm, m->xa, m->efmt, lm_rows, H, H, TC_BOX_A);
            if (lsplit) tc_make_map(&a_lm_lo, m->xa_lo, m->efmt, lm_rows, H, H, TC_BOX_A);
            launch_rows_to_half(m->efmt, m->h + static_cast<size_t>(lm_first) * H, H, lm_rows, H, m->final_norm, eps,
                                m->xa, lsplit ? m->xa_lo : nullptr, H, st);
            launch_gemm_tc(m->efmt, a_lm, lsplit ? &a_lm_lo : nullptr, m->tm_lm, lm_rows, m->v_loc, H, m->logits,
                           m->v_loc, LIN_STORE, false, nullptr, m->ctx->ws(), TC_WS_FLOATS, err, st);
        } else {
            launch_linear(m->efmt, m->lm_head, nullptr, m->v_loc, H, m->h + static_cast<size_t>(lm_first) * H, H,
                          lm_rows, m->final_norm, eps, m->logits, m->v_loc, LIN_STORE, st);
        }
        if (m->tp_size == 1) {
            launch_argmax(m->logits, m->v_loc, m->v_loc, lm_rows, m->temperature, m->d_keys, m->d_next, st);
        } else {
            unsigned long long* mine = m->d_keys + static_cast<size_t>(m->tp_rank) * lm_rows;
            launch_argmax_keys(m->logits, m->v_loc, m->v_loc, lm_rows, m->v_off, m->temperature, mine, st);
            nccl_check(nccl().all_gather(mine, m->d_keys, lm_rows, ncclUint64, m->comm, st), "argmax all-gather");
            launch_argmax_merge(m->d_keys, m->tp_size, lm_rows, m->d_next, st);
        }
    }
}

void check_ids(const soc_model* m, const int32_t* ids, int n) {
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || static_cast<size_t>(ids[i]) >= m->cfg.vocab)
            throw Error(SOC_B200_ERR_RANGE, "embedding input token id out of range");
}

// Copies the logits of `rows` rows (full vocab) to host memory.  With tensor parallelism
// the vocab shards are all-gathered first, so every rank must make the same call.
// All-gathers the vocab shards of `rows` logits rows into m->logits_all ([tp][rows][v_loc]).
void gather_logits(soc_model* m, int rows, cudaStream_t st) {
    const size_t V = m->cfg.vocab, vl = static_cast<size_t>(m->v_loc);
    if (rows > m->logits_all_rows) {
        m->dfree(m->logits_all);
        m->logits_all = static_cast<float*>(m->dmalloc(sizeof(float) * rows * V));
        m->logits_all_rows = rows;
    }
    nccl_check(nccl().all_gather(m->logits, m->logits_all, vl * rows, ncclFloat32, m->comm, st), "logits all-gather");
}

void logits_to_host(soc_model* m, int rows, float* host, cudaStream_t st) {
    const size_t V = m->cfg.vocab, vl = static_cast<size_t>(m->v_loc);
    if (m->tp_size == 1) {
        SOCB_CUDA(cudaMemcpyAsync(host, m->logits, sizeof(float) * V * rows, cudaMemcpyDeviceToHost, st));
        return;
    }
    gather_logits(m, rows, st);
    for (int r = 0; r < m->tp_size; ++r)
        SOCB_CUDA(cudaMemcpy2DAsync(host + r * vl, V * sizeof(float), m->logits_all + r * vl * rows, vl * sizeof(float),
                                    vl * sizeof(float), rows, cudaMemcpyDeviceToHost, st));
}

constexpr int kPrefillChunk = 4096;
constexpr int kPrefillGraphRows = 64;  // prefill chunks up to this many rows run as a cached graph

// SOC_B200_PREFILL_GRAPH=0 launches short prefill chunks directly instead of through a cached graph.
bool prefill_graph_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("SOC_B200_PREFILL_GRAPH");
        return !(e && std::string(e) == "0");
    }();
    return on;
}

// One prefill chunk (rows in m->d_tokens / d_seq / d_pos already) through a CUDA graph of its
// whole forward, captured on first use and replayed while the chunk's shape, cache slot,
// position and buffers stay the same (a generation job's prompt, over and over).  The values the
// kernels take as arguments (flash attention's start, the last-row lm_head) are in the key.
void prefill_graph(soc_model* m, soc_kv* kv, int seq, int start, int n, bool last) {
    cudaStream_t st = m->ctx->stream;
    // everything the forward allocates lazily is allocated before a capture
    ensure_logits(m, 1);
    if (m->tc_ok) m->ctx->ws();
    const soc_model::PrefillKey key{kv, m->h, m->xa, m->logits, m->buf_epoch, seq, start, n, last ? 1 : 0,
                                    m->temperature};
    if (!m->pf_graph || !(m->pf_key == key)) {
        if (m->pf_graph) cudaGraphExecDestroy(m->pf_graph);
        m->pf_graph = nullptr;
        cudaGraph_t g = nullptr;
        const long long before = launches_so_far();
        SOCB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        try {
            forward_rows(m, kv, n, start + n, last ? n - 1 : 0, last ? 1 : 0, 1, seq, start);
        } catch (...) {
            cudaStreamEndCapture(st, &g);
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            count_launches(-(launches_so_far() - before));
            m->pf_graph_broken = true;
            forward_rows(m, kv, n, start + n, last ? n - 1 : 0, last ? 1 : 0, 1, seq, start);
            return;
        }
        m->pf_graph_kernels = launches_so_far() - before;
        count_launches(-(launches_so_far() - before));
        SOCB_CUDA(cudaStreamEndCapture(st, &g));
        const cudaError_t e = cudaGraphInstantiate(&m->pf_graph, g, 0);
        cudaGraphDestroy(g);
        SOCB_CUDA(e);
        m->pf_key = key;
        m->pf_key.epoch = m->buf_epoch;
    }
    SOCB_CUDA(cudaGraphLaunch(m->pf_graph, st));
    count_launches(m->pf_graph_kernels);
}

// Prefill `n` host ids at the end of `seq`; leaves the last row's logits/next id on the device.
void prefill_impl(soc_model* m, soc_kv* kv, int seq, const int32_t* ids, int n, bool ids_on_device) {
    kv->check_seq(seq);
    if (n <= 0) throw Error(SOC_B200_ERR_INVALID, "GenerationContext prefill requires at least one token");
    if (!ids_on_device) check_ids(m, ids, n);
    cudaStream_t st = m->ctx->stream;
    const int start = kv->lengths[seq];
    kv->reserve(seq, start + n, st);
    for (int off = 0; off < n; off += kPrefillChunk) {
        const int cn = std::min(kPrefillChunk, n - off);
        ensure_workspace(m, cn);
        std::vector<int> sq(cn, seq), ps(cn);
        for (int i = 0; i < cn; ++i) ps[i] = start + off + i;
        SOCB_CUDA(cudaMemcpyAsync(m->d_tokens, ids + off, sizeof(int) * cn,
                                  ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
        SOCB_CUDA(cudaMemcpyAsync(m->d_seq, sq.data(), sizeof(int) * cn, cudaMemcpyHostToDevice, st));
        SOCB_CUDA(cudaMemcpyAsync(m->d_pos, ps.data(), sizeof(int) * cn, cudaMemcpyHostToDevice, st));
        const bool last = off + cn == n;
        // (the pageable host vectors are staged by the driver before cudaMemcpyAsync returns)
        if (m->tp_size == 1 && cn <= kPrefillGraphRows && !m->pf_graph_broken && prefill_graph_enabled())
            prefill_graph(m, kv, seq, start + off, cn, last);
        else
            forward_rows(m, kv, cn, start + off + cn, last ? cn - 1 : 0, last ? 1 : 0, 1, seq, start + off);
    }
    kv->lengths[seq] = start + n;
}


__global__ void k_step_begin(const soc_model::LoopState* st, int* tokens, int* seq, int* pos) {
    const int i = st->step;
    tokens[0] = st->out[i];
    seq[0] = st->seq;
    pos[0] = st->start + i;
}

__global__ void k_step_end(soc_model::LoopState* st, const int* next) {
    st->out[st->step + 1] = next[0];
    st->step += 1;
}

__device__ __forceinline__ unsigned loop_continues(const soc_model::LoopState* st) {
    const int s = st->step;
    return (s < st->steps && !(st->eos >= 0 && st->out[s] == st->eos)) ? 1u : 0u;
}

// Before the loop: whether its first step runs (the generation context stops on an EOS input).
__global__ void k_loop_gate(const soc_model::LoopState* st, cudaGraphConditionalHandle h) {
    cudaGraphSetConditional(h, loop_continues(st));
}

// End of a step inside the loop: record the id, then whether the next step runs.  The step
// counter grows by one per iteration and the loop ends at st->steps, so it always ends.
__global__ void k_step_end_loop(soc_model::LoopState* st, const int* next, cudaGraphConditionalHandle h) {
    st->out[st->step + 1] = next[0];
    st->step += 1;
    cudaGraphSetConditional(h, loop_continues(st));
}

// Parameters of one persistent-kernel launch (decode_mk.cu) over the buffers given.
MKParams mk_params(const soc_model* m, const soc_kv* kv, int seq, int start, int steps, int* d_ids, float* logits,
                   int eos, int splits, int group, unsigned long long* vec, unsigned long long* part,
                   unsigned long long* best,
                   unsigned tag0) {
    const Config& c = m->cfg;
    MKParams p{};
    p.L = static_cast<int>(c.layers);
    p.H = static_cast<int>(c.hidden);
    p.I = static_cast<int>(c.inter);
    p.hq = static_cast<int>(c.hq);
    p.hkv = static_cast<int>(c.hkv);
    p.D = static_cast<int>(c.hd);
    p.V = static_cast<int>(c.vocab);
    p.eps = static_cast<float>(c.eps);
    p.wfmt = m->wfmt;
    p.efmt = m->efmt;
    p.layers = m->d_mk_layers;
    p.embed = m->embed;
    p.lm_tiles = m->mk_lm_tiles;
    p.final_norm = m->final_norm;
    p.rope_cs = m->rope_cs;
    p.rope_len = m->rope_len;
    p.kpool = kv->k;
    p.vpool = kv->v;
    p.kv_layer_stride = kv->layer_stride();
    p.page_table = kv->d_page_table + static_cast<size_t>(seq) * kv->max_pages;
    p.page_tokens = kv->page_tokens;
    p.max_pages = kv->max_pages;
    p.ids = d_ids;
    p.start = start;
    p.steps = steps;
    p.logits = logits;
    p.temperature = m->temperature;
    p.eos = eos;
    p.vec = vec;
    p.part = part;
    p.tag0 = tag0;
    p.best = best;
    p.err = m->ctx->d_err;
    p.att_splits = splits;
    p.att_group = group;
    // ring chunks in flight (SOC_B200_MK_INFLIGHT, default 2)
    static const int inflight = [] {
        const char* e = std::getenv("SOC_B200_MK_INFLIGHT");
        const int v = e && *e ? std::atoi(e) : 2;
        return std::max(1, std::min(v, 4));
    }();
    p.inflight = inflight;
    p.trace = nullptr;
    return p;
}

// Tag base for a launch of `steps` steps on tagged buffers whose last launch ended at *tag:
// tags only grow, and before they would wrap the buffers are cleared and counting restarts
// (a stale word must never carry a tag a reader waits for).
unsigned mk_next_tags(unsigned* tag, int steps, int L, unsigned long long* vec, size_t vec_n,
                      unsigned long long* part, size_t part_n, cudaStream_t st) {
    const unsigned long long need = mk_tags_per_launch(steps, L);
    if (static_cast<unsigned long long>(*tag) + need >= 0xF0000000ull) {
        SOCB_CUDA(cudaMemsetAsync(vec, 0, vec_n * sizeof(unsigned long long), st));
        if (part_n) SOCB_CUDA(cudaMemsetAsync(part, 0, part_n * sizeof(unsigned long long), st));
        *tag = 0;
    }
    const unsigned base = *tag;
    *tag = static_cast<unsigned>(base + need);
    return base;
}

// Persistent-kernel decode of `steps` tokens of one sequence (see decode_mk.cu).
void run_mk(soc_model* m, soc_kv* kv, int seq, int start, int steps, int* d_ids, float* logits, int eos = -1) {
    const Config& c = m->cfg;
    cudaStream_t st = m->ctx->stream;
    if (start + steps > m->rope_len) throw Error(SOC_B200_ERR_CAPACITY, "decode position beyond the RoPE table");
    ensure_workspace(m, 16);
    const int hkv = static_cast<int>(c.hkv);
    if (steps > m->mk_best_n) {
        m->dfree(m->mk_best);
        m->mk_best_n = std::max(steps, 64);
        m->mk_best = static_cast<unsigned long long*>(
            m->dmalloc(sizeof(unsigned long long) * m->mk_best_n * m->mk_grid));
    }
    int group = 1;
    const int S = mk_att_plan(start + steps, static_cast<int>(c.hq), hkv, m->mk_grid, &group);
    const size_t part = S > 1 ? mk_part_words(static_cast<int>(c.hq), hkv, static_cast<int>(c.hd), S) : 0;
    if (part > m->mk_part_n) {
        // a new buffer starts zeroed: no stale tags
        m->dfree(m->mk_part);
        m->mk_part = static_cast<unsigned long long*>(m->dmalloc(sizeof(unsigned long long) * part));
        SOCB_CUDA(cudaMemsetAsync(m->mk_part, 0, sizeof(unsigned long long) * part, st));
        m->mk_part_n = part;
    }
    SOCB_CUDA(cudaMemsetAsync(m->mk_best, 0, sizeof(unsigned long long) * steps * m->mk_grid, st));
    const unsigned tag0 = mk_next_tags(&m->mk_tag, steps, static_cast<int>(c.layers), m->mk_vec, m->mk_vec_n,
                                       m->mk_part, m->mk_part_n, st);
    MKParams p =
        mk_params(m, kv, seq, start, steps, d_ids, logits, eos, S, group, m->mk_vec, m->mk_part, m->mk_best, tag0);
    // Optional phase trace (SOC_B200_MK_TRACE=<file>): raw u64 %globaltimer stamps of the first step.
    const char* trace_path = std::getenv("SOC_B200_MK_TRACE");
    unsigned long long* trace = nullptr;
    const size_t trace_n = static_cast<size_t>(m->mk_grid) * mk_trace_stride(static_cast<int>(c.layers));
    if (trace_path && *trace_path) {
        trace = static_cast<unsigned long long*>(m->dmalloc(trace_n * sizeof(unsigned long long)));
        SOCB_CUDA(cudaMemsetAsync(trace, 0, trace_n * sizeof(unsigned long long), st));
    }
    p.trace = trace;
    mk_launch(p, m->mk_grid, st);
    count_launches(1);
    if (trace) {
        std::vector<unsigned long long> host(trace_n);
        SOCB_CUDA(cudaMemcpyAsync(host.data(), trace, trace_n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, st));
        SOCB_CUDA(cudaStreamSynchronize(st));
        m->dfree(trace, false);
        if (FILE* f = std::fopen(trace_path, "wb")) {
            const int hdr[4] = {m->mk_grid, static_cast<int>(c.layers), MK_TRACE_PER_LAYER, steps};
            std::fwrite(hdr, sizeof(int), 4, f);
            std::fwrite(host.data(), sizeof(unsigned long long), trace_n, f);
            std::fclose(f);
        }
    }
}

// `steps` decode steps of sequence `seq`, whose cache holds `start` tokens and whose
// next input id is d_out[0]; writes ids 1..steps of d_out.  Without the persistent kernel the
// loop is one CUDA graph (bound to this cache, split count and buffers): a WHILE node around one
// captured step.  eos >= 0: both stop on the device at the first step whose input id is eos (ids
// after it are not written); the tensor-parallel path (collectives stay out of graphs) runs every
// step.
void decode_loop(soc_model* m, soc_kv* kv, int seq, int start, int steps, int32_t* d_out, int eos = -1) {
    if (m->mk_ok) {
        run_mk(m, kv, seq, start, steps, d_out, nullptr, eos);
        return;
    }
    cudaStream_t st = m->ctx->stream;
    const int splits = attention_splits(1, static_cast<int>(m->cfg.hkv), start + steps);
    ensure_workspace(m, 1);
    ensure_logits(m, 1);
    if (splits > 1) ensure_attn_scratch(m, static_cast<size_t>(m->cfg.hq) * splits * (m->cfg.hd + 2));
    if (!m->d_loop) m->d_loop = static_cast<soc_model::LoopState*>(m->dmalloc(sizeof(soc_model::LoopState)));
    if (m->tp_size > 1) {
        // Tensor-parallel steps are queued one by one (their collectives stay out of graphs).
        const soc_model::LoopState init{d_out, seq, start, 0, steps, -1};
        SOCB_CUDA(cudaMemcpyAsync(m->d_loop, &init, sizeof(init), cudaMemcpyHostToDevice, st));
        for (int i = 0; i < steps; ++i) {
            k_step_begin<<<1, 1, 0, st>>>(m->d_loop, m->d_tokens, m->d_seq, m->d_pos);
            forward_rows(m, kv, 1, start + steps, 0, 1, splits);
            k_step_end<<<1, 1, 0, st>>>(m->d_loop, m->d_next);
            count_launches(2);
        }
        return;
    }
    if (!m->step_graph || m->graph_kv != kv || m->graph_splits != splits || m->graph_epoch != m->buf_epoch) {
        // One graph runs the whole loop: a gate kernel, then a WHILE node whose body is one
        // decode step ending in the kernel that decides whether the next step runs.
        if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
        m->step_graph = nullptr;
        cudaGraph_t g = nullptr, tmp = nullptr;
        SOCB_CUDA(cudaGraphCreate(&g, 0));
        const long long before = launches_so_far();
        try {
            cudaGraphConditionalHandle h{};
            SOCB_CUDA(cudaGraphConditionalHandleCreate(&h, g, 0, 0));
            SOCB_CUDA(cudaStreamBeginCaptureToGraph(st, g, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
            k_loop_gate<<<1, 1, 0, st>>>(m->d_loop, h);
            SOCB_CUDA(cudaStreamEndCapture(st, &tmp));
            cudaGraphNode_t gate = nullptr;
            size_t nn = 1;
            SOCB_CUDA(cudaGraphGetNodes(g, &gate, &nn));
            cudaGraphNodeParams cp{};
            cp.type = cudaGraphNodeTypeConditional;
            cp.conditional.handle = h;
            cp.conditional.type = cudaGraphCondTypeWhile;
            cp.conditional.size = 1;
            cudaGraphNode_t loop = nullptr;
            SOCB_CUDA(cudaGraphAddNode(&loop, g, &gate, 1, &cp));
            const cudaGraph_t body = cp.conditional.phGraph_out[0];
            SOCB_CUDA(cudaStreamBeginCaptureToGraph(st, body, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
            try {
                k_step_begin<<<1, 1, 0, st>>>(m->d_loop, m->d_tokens, m->d_seq, m->d_pos);
                forward_rows(m, kv, 1, start + steps, 0, 1, splits);
                k_step_end_loop<<<1, 1, 0, st>>>(m->d_loop, m->d_next, h);
            } catch (...) {
                cudaStreamEndCapture(st, &tmp);
                throw;
            }
            SOCB_CUDA(cudaStreamEndCapture(st, &tmp));
            // captured launches did not run: move them from the counter to the graph's size
            m->graph_kernels = launches_so_far() - before + 2;
            count_launches(-(launches_so_far() - before));
            SOCB_CUDA(cudaGraphInstantiate(&m->step_graph, g, 0));
        } catch (...) {
            count_launches(-(launches_so_far() - before));
            cudaGraphDestroy(g);
            cudaGetLastError();
            throw;
        }
        cudaGraphDestroy(g);
        m->graph_kv = kv;
        m->graph_splits = splits;
        m->graph_epoch = m->buf_epoch;
    }
    const soc_model::LoopState init{d_out, seq, start, 0, steps, eos};
    SOCB_CUDA(cudaMemcpyAsync(m->d_loop, &init, sizeof(init), cudaMemcpyHostToDevice, st));
    SOCB_CUDA(cudaGraphLaunch(m->step_graph, st));
    // counted as if every step runs; soc_b200_generate corrects the count after an EOS stop
    count_launches(1 + m->graph_kernels * steps);
    m->loop_steps_queued = steps;
}

}  // namespace

// ============================================================== C ABI
extern "C" {

const char* soc_b200_last_error(void) { return g_last_error.c_str(); }

long long soc_b200_kernel_launches(void) { return launches_so_far(); }

int soc_b200_open(int device, soc_ctx** out) {
    if (!out) return fail(SOC_B200_ERR_INVALID, "soc_b200_open: null output");
    return guarded([&] {
        int n = 0;
        SOCB_CUDA(cudaGetDeviceCount(&n));
        if (device < 0 || device >= n) throw Error(SOC_B200_ERR_INVALID, "soc_b200_open: device index out of range");
        SOCB_CUDA(cudaSetDevice(device));
        auto c = std::make_unique<soc_ctx>();
        c->device = device;
        SOCB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        SOCB_CUDA(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device));
        SOCB_CUDA(cudaMalloc(&c->d_err, sizeof(int)));
        SOCB_CUDA(cudaMemset(c->d_err, 0, sizeof(int)));
        *out = c.release();
    });
}

void soc_b200_close(soc_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_err);
    if (ctx->lin_scratch) cudaFree(ctx->lin_scratch);
    if (ctx->gemm_ws) cudaFree(ctx->gemm_ws);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
}

int soc_b200_synchronize(soc_ctx* ctx) {
    if (!ctx) return fail(SOC_B200_ERR_INVALID, "null context");
    return guarded([&] { SOCB_CUDA(cudaStreamSynchronize(ctx->stream)); });
}

void* soc_b200_stream(soc_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int soc_b200_load_bundle(soc_ctx* ctx, const char* manifest_path, int weight_format, int tp_rank, int tp_size,
                         void* nccl_comm, soc_model** out) {
    if (!ctx || !manifest_path || !out) return fail(SOC_B200_ERR_INVALID, "soc_b200_load_bundle: null argument");
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size)
        return fail(SOC_B200_ERR_INVALID, "soc_b200_load_bundle: tp_rank must be in [0, tp_size)");
    if (tp_size > 1 && nccl_comm == nullptr)
        return fail(SOC_B200_ERR_INVALID, "soc_b200_load_bundle: tensor parallelism needs an NCCL communicator");
    auto m = std::make_unique<soc_model>();
    int rc = guarded([&] {
        SOCB_CUDA(cudaSetDevice(ctx->device));
        m->ctx = ctx;
        const Manifest man = load_manifest(manifest_path);
        m->cfg_full = read_config(man.config);
        m->cfg = m->cfg_full;
        m->tp_rank = tp_rank;
        m->tp_size = tp_size;
        m->comm = static_cast<ncclComm_t>(nccl_comm);
        if (tp_size > 1) {
            const Config& f = m->cfg_full;
            if (f.hq % tp_size || f.hkv % tp_size || f.inter % tp_size || f.vocab % tp_size)
                throw Error(SOC_B200_ERR_INVALID,
                            "tensor parallelism needs heads, kv heads, intermediate size and vocab divisible by tp_size");
            if ((f.inter / tp_size) % 64 || (f.hq / tp_size * f.hd) % 64)
                throw Error(SOC_B200_ERR_INVALID, "tensor-parallel shards must keep multiples of 64 features");
            m->cfg.hq /= tp_size;
            m->cfg.hkv /= tp_size;
            m->cfg.inter /= tp_size;
        }
        const Config& c = m->cfg;
        const size_t H = c.hidden, I = c.inter, D = c.hd, QW = c.hq * D, KW = c.hkv * D;
        const size_t QWf = m->cfg_full.hq * D, KWf = m->cfg_full.hkv * D, If = m->cfg_full.inter;
        const size_t tr = static_cast<size_t>(tp_rank);
        m->v_loc = static_cast<int>(c.vocab / tp_size);
        m->v_off = static_cast<int>(tr * m->v_loc);

        // Linear weight format: the stored type of the block linears unless the caller asks
        // for another one (float -> float conversion, or group quantisation at load time).
        const std::string lin_dtype = man.find("model.layers.0.self_attn.q_proj.weight").dtype;
        int fmt = fmt_of_dtype(lin_dtype);
        if (fmt == 0) throw_fmt("model loader requires floating-point weights for: model.layers.0.self_attn.q_proj.weight");
        if (weight_format == SOC_B200_WEIGHTS_F16) fmt = WF_F16;
        else if (weight_format == SOC_B200_WEIGHTS_BF16) fmt = WF_BF16;
        else if (weight_format == SOC_B200_WEIGHTS_INT8_G64) fmt = WF_I8G64;
        else if (weight_format == SOC_B200_WEIGHTS_INT4_G32) fmt = WF_I4G32;
        else if (weight_format != SOC_B200_WEIGHTS_NATIVE)
            throw Error(SOC_B200_ERR_INVALID, "soc_b200_load_bundle: unknown weight_format");
        m->wfmt = fmt;
        const bool quant = quant_group(fmt) != 0;

        // Converts a float tensor to the device element type `f` (bit copy when it already matches).
        auto upload_matrix = [&](const TensorRecord& r, const std::vector<char>& b, void* dst, int f) {
            const size_t n = b.size() / dtype_width(r.dtype);
            const bool same = (f == WF_F16 && r.dtype == "float16") || (f == WF_BF16 && r.dtype == "bfloat16");
            if (same) {
                SOCB_CUDA(cudaMemcpy(dst, b.data(), b.size(), cudaMemcpyHostToDevice));
                return;
            }
            const std::vector<float> fv = to_f32(r, b);
            std::vector<uint16_t> conv(n);
            for (size_t i = 0; i < n; ++i) {
                if (f == WF_F16) {
                    conv[i] = float_to_half_bits(fv[i]);
                } else {
                    const __nv_bfloat16 bb = __float2bfloat16_rn(fv[i]);
                    std::memcpy(&conv[i], &bb, 2);
                }
            }
            SOCB_CUDA(cudaMemcpy(dst, conv.data(), n * 2, cudaMemcpyHostToDevice));
        };
        auto upload_norm = [&](const std::string& name, size_t n) -> float* {
            const TensorRecord& r = man.find(name);
            const std::vector<float> f = to_f32(r, load_record(r, {n}));
            float* d = static_cast<float*>(m->dmalloc(n * sizeof(float)));
            SOCB_CUDA(cudaMemcpy(d, f.data(), n * sizeof(float), cudaMemcpyHostToDevice));
            return d;
        };

        // Embedding (and tied lm_head).
        {
            const TensorRecord& r = man.find("model.embed_tokens.weight");
            const auto b = load_record(r, {c.vocab, H});
            m->efmt = r.dtype == "bfloat16" ? WF_BF16 : WF_F16;
            if (weight_format == SOC_B200_WEIGHTS_BF16) m->efmt = WF_BF16;
            if (weight_format == SOC_B200_WEIGHTS_F16) m->efmt = WF_F16;
            m->embed = m->dmalloc(c.vocab * H * 2);
            upload_matrix(r, b, m->embed, m->efmt);
        }
        m->layers.resize(c.layers);
        for (size_t l = 0; l < c.layers; ++l) {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            LayerW& w = m->layers[l];
            w.in_norm = upload_norm(p + "input_layernorm.weight", H);
            w.post_norm = upload_norm(p + "post_attention_layernorm.weight", H);
            w.q_norm = upload_norm(p + "self_attn.q_norm.weight", D);
            w.k_norm = upload_norm(p + "self_attn.k_norm.weight", D);
            // Uploads rows of one or more matrices (concatenated, or interleaved row by row).
            auto upload_rows = [&](const std::vector<HostMat>& mats, const std::vector<size_t>& rows, size_t cols,
                                   bool interleave, void** dst, void** sdst) {
                const size_t rb = fmt_row_bytes(fmt, cols), sr = quant ? cols / quant_group(fmt) : 0;
                size_t total = 0;
                for (size_t r : rows) total += r;
                std::vector<uint8_t> data(total * rb);
                std::vector<uint16_t> sc(total * sr);
                if (!interleave) {
                    size_t at = 0;
                    for (size_t i = 0; i < mats.size(); ++i) {
                        std::memcpy(data.data() + at * rb, mats[i].data.data(), rows[i] * rb);
                        if (quant) std::memcpy(sc.data() + at * sr, mats[i].scales.data(), rows[i] * sr * 2);
                        at += rows[i];
                    }
                } else {  // rows (2j, 2j+1) = (mats[0] row j, mats[1] row j)
                    for (size_t j = 0; j < rows[0]; ++j)
                        for (int t = 0; t < 2; ++t) {
                            std::memcpy(data.data() + (2 * j + t) * rb, mats[t].data.data() + j * rb, rb);
                            if (quant)
                                std::memcpy(sc.data() + (2 * j + t) * sr, mats[t].scales.data() + j * sr, sr * 2);
                        }
                }
                *dst = m->dmalloc(data.size());
                SOCB_CUDA(cudaMemcpy(*dst, data.data(), data.size(), cudaMemcpyHostToDevice));
                if (quant) {
                    *sdst = m->dmalloc(sc.size() * 2);
                    SOCB_CUDA(cudaMemcpy(*sdst, sc.data(), sc.size() * 2, cudaMemcpyHostToDevice));
                }
            };
            // this rank's shard: rows of q/k/v and gate/up, columns of o_proj and down_proj
            upload_rows({prepare_matrix(man, p + "self_attn.q_proj.weight", QWf, H, fmt, Block{tr * QW, QW, 0, H}),
                         prepare_matrix(man, p + "self_attn.k_proj.weight", KWf, H, fmt, Block{tr * KW, KW, 0, H}),
                         prepare_matrix(man, p + "self_attn.v_proj.weight", KWf, H, fmt, Block{tr * KW, KW, 0, H})},
                        {QW, KW, KW}, H, false, &w.wqkv, &w.sqkv);
            upload_rows({prepare_matrix(man, p + "self_attn.o_proj.weight", H, QWf, fmt, Block{0, H, tr * QW, QW})}, {H},
                        QW, false, &w.wo, &w.so);
            upload_rows({prepare_matrix(man, p + "mlp.gate_proj.weight", If, H, fmt, Block{tr * I, I, 0, H}),
                         prepare_matrix(man, p + "mlp.up_proj.weight", If, H, fmt, Block{tr * I, I, 0, H})},
                        {I, I}, H, true, &w.wgu, &w.sgu);
            upload_rows({prepare_matrix(man, p + "mlp.down_proj.weight", H, If, fmt, Block{0, H, tr * I, I})}, {H}, I,
                        false, &w.wd, &w.sd);
        }
        m->final_norm = upload_norm("model.norm.weight", H);
        // TMA descriptors of the block linears for the tensor-core GEMM (for quantised
        // models: of the fp16 expansion buffer, one per matrix shape).
        m->tc_ok = tc_available();
        m->gfmt = fmt == WF_BF16 ? WF_BF16 : WF_F16;
        if (m->tc_ok && !quant) {
            for (auto& w : m->layers) {
                tc_make_map(&w.tm_qkv, w.wqkv, fmt, QW + 2 * KW, H, H, TC_BOX_W);
                tc_make_map(&w.tm_o, w.wo, fmt, H, QW, QW, TC_BOX_W);
                tc_make_map(&w.tm_gu, w.wgu, fmt, 2 * I, H, H, TC_BOX_W);
                tc_make_map(&w.tm_d, w.wd, fmt, H, I, I, TC_BOX_W);
            }
        } else if (m->tc_ok) {
            const size_t most = std::max({(QW + 2 * KW) * H, H * QW, 2 * I * H, H * I});
            m->wdq = m->dmalloc(most * 2);
            tc_make_map(&m->tm_dq_qkv, m->wdq, WF_F16, QW + 2 * KW, H, H, TC_BOX_W);
            tc_make_map(&m->tm_dq_o, m->wdq, WF_F16, H, QW, QW, TC_BOX_W);
            tc_make_map(&m->tm_dq_gu, m->wdq, WF_F16, 2 * I, H, H, TC_BOX_W);
            tc_make_map(&m->tm_dq_d, m->wdq, WF_F16, H, I, I, TC_BOX_W);
        }
        // lm_head rows [v_off, v_off + v_loc) (all of them without tensor parallelism)
        const size_t vl = static_cast<size_t>(m->v_loc), vo = static_cast<size_t>(m->v_off);
        if (c.tied && tp_size == 1) {
            m->lm_head = m->embed;
        } else {
            const TensorRecord& r = man.find(c.tied ? "model.embed_tokens.weight" : "lm_head.weight");
            std::vector<char> b = load_record(r, {c.vocab, H});
            const size_t rb = H * dtype_width(r.dtype);
            if (tp_size > 1) b = std::vector<char>(b.begin() + vo * rb, b.begin() + (vo + vl) * rb);
            m->lm_head = m->dmalloc(vl * H * 2);
            upload_matrix(r, b, m->lm_head, m->efmt);
        }
        if (m->tc_ok && (m->efmt == WF_F16 || m->efmt == WF_BF16))
            tc_make_map(&m->tm_lm, m->lm_head, m->efmt, static_cast<uint64_t>(m->v_loc), H, H, TC_BOX_W);
        else
            m->tc_ok = false;
        // RoPE table (cos, sin) [max_pos][D/2], computed as RoPE::ApplyInPlace does (rope.cpp:74-79).
        m->rope_len = static_cast<int>(c.max_pos);
        std::vector<float2> cs(static_cast<size_t>(m->rope_len) * (D / 2));
        for (int pos = 0; pos < m->rope_len; ++pos) {
            const double ap = static_cast<double>(pos);
            for (size_t i = 0; i < D / 2; ++i) {
                const double ex = static_cast<double>(i * 2) / static_cast<double>(D);
                const double ang = ap / std::pow(c.theta, ex);
                cs[static_cast<size_t>(pos) * (D / 2) + i] =
                    make_float2(static_cast<float>(std::cos(ang)), static_cast<float>(std::sin(ang)));
            }
        }
        m->rope_cs = static_cast<float2*>(m->dmalloc(cs.size() * sizeof(float2)));
        SOCB_CUDA(cudaMemcpy(m->rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice));
        ensure_workspace(m.get(), 16);
        // Persistent decode kernel, unless the shape is outside its limits or the
        // caller asks for the graph path (SOC_B200_DECODE_PATH=graph).
        const char* path = std::getenv("SOC_B200_DECODE_PATH");
        const bool want_mk = !(path && std::string(path) == "graph");
        const int grid = mk_grid(ctx->device);
        if (want_mk && tp_size == 1 &&
            mk_supported(static_cast<int>(c.layers), static_cast<int>(H), static_cast<int>(I), static_cast<int>(c.hq), static_cast<int>(c.hkv),
                         static_cast<int>(D), static_cast<int>(c.vocab), fmt, m->efmt, grid)) {
            // the kernel's own copy of every matrix, in its tiled layout (the row-major copies
            // stay for prefill and batched decode)
            const int Hi = static_cast<int>(H), Ii = static_cast<int>(I), QKVr = static_cast<int>(QW + 2 * KW);
            const int QWi = static_cast<int>(QW);
            auto tiled = [&](const void* w, const void* sc, int rows, int K, int f) -> void* {
                void* d = m->dmalloc(mk_tiled_bytes(f, rows, K));
                mk_tile_matrix(f, w, sc, rows, K, d, ctx->stream);
                return d;
            };
            std::vector<MKLayer> ml(c.layers);
            for (size_t l = 0; l < c.layers; ++l) {
                const LayerW& w = m->layers[l];
                ml[l] = MKLayer{tiled(w.wqkv, w.sqkv, QKVr, Hi, fmt), tiled(w.wo, w.so, Hi, QWi, fmt),
                                tiled(w.wgu, w.sgu, 2 * Ii, Hi, fmt),  tiled(w.wd, w.sd, Hi, Ii, fmt),
                                w.in_norm, w.post_norm, w.q_norm, w.k_norm};
            }
            m->mk_lm_tiles = tiled(m->lm_head, nullptr, static_cast<int>(c.vocab), Hi, m->efmt);
            m->d_mk_layers = static_cast<MKLayer*>(m->dmalloc(sizeof(MKLayer) * c.layers));
            SOCB_CUDA(cudaMemcpy(m->d_mk_layers, ml.data(), sizeof(MKLayer) * c.layers, cudaMemcpyHostToDevice));
            m->mk_ids = static_cast<int*>(m->dmalloc(sizeof(int) * 2));
            m->mk_vec_n = mk_vec_words(Hi, Ii, static_cast<int>(c.hq), static_cast<int>(c.hkv), static_cast<int>(D));
            m->mk_vec = static_cast<unsigned long long*>(m->dmalloc(sizeof(unsigned long long) * m->mk_vec_n));
            SOCB_CUDA(cudaMemset(m->mk_vec, 0, sizeof(unsigned long long) * m->mk_vec_n));
            m->mk_grid = grid;
            m->mk_ok = true;
        }
        SOCB_CUDA(cudaDeviceSynchronize());
    });
    // Peer-memory all-reduce for decode-sized steps (up to 64 rows), last because setting it
    // up is collective: every rank comes here whether or not its load succeeded, and the
    // ranks agree on success before each collective step, so one rank's failed load makes
    // every rank's load fail instead of leaving the others waiting in NCCL.
    if (tp_size > 1 && tp_p2p_requested()) {
        const bool load_ok = rc == SOC_B200_OK;
        const std::string load_err = load_ok ? std::string() : std::string(soc_b200_last_error());
        const int rc2 = guarded([&] {
            SOCB_CUDA(cudaSetDevice(ctx->device));
            m->ar = new TpExchange();
            m->ar->setup(static_cast<ncclComm_t>(nccl_comm), tp_rank, tp_size,
                         static_cast<size_t>(64) * m->cfg.hidden, load_ok, ctx->stream);
        });
        if (!load_ok)
            fail(rc, load_err);  // the load's own error is the one to report
        else
            rc = rc2;
    }
    if (rc != SOC_B200_OK) {
        if (m->ar) {
            m->ar->release();
            delete m->ar;
        }
        for (void* p : m->allocs)
            if (p) cudaFree(p);
        return rc;
    }
    *out = m.release();
    return SOC_B200_OK;
}

int soc_b200_validate_bundle(const char* manifest_path) {
    if (!manifest_path) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] { validate_bundle(manifest_path); });
}

int soc_b200_model_info(const soc_model* m, soc_model_info* out) {
    if (!m || !out) return fail(SOC_B200_ERR_INVALID, "null argument");
    const Config& c = m->cfg_full;
    out->layers = static_cast<int>(c.layers);
    out->hidden = static_cast<int>(c.hidden);
    out->intermediate = static_cast<int>(c.inter);
    out->q_heads = static_cast<int>(c.hq);
    out->kv_heads = static_cast<int>(c.hkv);
    out->head_dim = static_cast<int>(c.hd);
    out->vocab = static_cast<int>(c.vocab);
    out->tied_embeddings = c.tied ? 1 : 0;
    out->weight_format = m->wfmt;
    out->max_position = m->rope_len;
    out->rms_norm_eps = static_cast<float>(c.eps);
    out->rope_theta = c.theta;
    out->tp_rank = m->tp_rank;
    out->tp_size = m->tp_size;
    return SOC_B200_OK;
}

int soc_b200_set_sampler(soc_model* m, float temperature, size_t top_k) {
    if (!m) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (!(temperature > 0.0f)) return fail(SOC_B200_ERR_INVALID, "sampler temperature must be positive");
    if (top_k == 0) return fail(SOC_B200_ERR_INVALID, "sampler top_k must be positive");
    return guarded([&] {
        if (temperature != m->temperature) {
            // the captured decode step holds the old temperature as a kernel argument
            SOCB_CUDA(cudaSetDevice(m->ctx->device));
            SOCB_CUDA(cudaStreamSynchronize(m->ctx->stream));
            if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
            m->step_graph = nullptr;
            m->graph_kv = nullptr;
            if (m->pf_graph) cudaGraphExecDestroy(m->pf_graph);
            m->pf_graph = nullptr;
        }
        m->temperature = temperature;
        m->top_k = top_k;
    });
}

void soc_b200_free_model(soc_model* m) {
    if (!m) return;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
    if (m->pf_graph) cudaGraphExecDestroy(m->pf_graph);
    if (m->ar) {
        m->ar->release();
        delete m->ar;
    }
    for (void* p : m->allocs)
        if (p) cudaFree(p);
    delete m;
}

int soc_b200_kv_create(soc_model* m, int max_seqs, int max_tokens, int page_tokens, soc_kv** out) {
    if (!m || !out) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (max_seqs <= 0 || max_tokens <= 0) return fail(SOC_B200_ERR_INVALID, "kv cache requires positive capacity");
    if (page_tokens != 16) return fail(SOC_B200_ERR_INVALID, "kv cache page_tokens must be 16");
    auto kv = std::make_unique<soc_kv>();
    const int rc = guarded([&] {
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        kv->m = m;
        kv->max_seqs = max_seqs;
        kv->page_tokens = page_tokens;
        kv->num_pages = (max_tokens + page_tokens - 1) / page_tokens;
        kv->max_pages = std::min(kv->num_pages, (m->rope_len + page_tokens - 1) / page_tokens);
        const size_t elems = static_cast<size_t>(m->cfg.layers) * kv->layer_stride();
        SOCB_CUDA(cudaMalloc(&kv->k, elems * sizeof(__half)));
        SOCB_CUDA(cudaMalloc(&kv->v, elems * sizeof(__half)));
        SOCB_CUDA(cudaMalloc(&kv->d_page_table, sizeof(int) * static_cast<size_t>(max_seqs) * kv->max_pages));
        {  // 2-D TMA views [L * pages * hkv * 16, head_dim] of the pools (row index must fit int32)
            const size_t rows = m->cfg.layers * static_cast<size_t>(kv->num_pages) * m->cfg.hkv * page_tokens;
            if (tc_available() && rows < (size_t(1) << 31) && m->cfg.hd % 64 == 0) {
                tc_make_map(&kv->tmk, kv->k, WF_F16, rows, m->cfg.hd, m->cfg.hd, static_cast<uint32_t>(page_tokens));
                tc_make_map(&kv->tmv, kv->v, WF_F16, rows, m->cfg.hd, m->cfg.hd, static_cast<uint32_t>(page_tokens));
                kv->tm_ok = true;
            }
        }
        SOCB_CUDA(cudaMemset(kv->d_page_table, 0, sizeof(int) * static_cast<size_t>(max_seqs) * kv->max_pages));
        kv->lengths.assign(max_seqs, 0);
        kv->pages.assign(max_seqs, {});
        kv->free_pages.resize(kv->num_pages);
        for (int i = 0; i < kv->num_pages; ++i) kv->free_pages[i] = kv->num_pages - 1 - i;
    });
    if (rc != SOC_B200_OK) {
        cudaFree(kv->k);
        cudaFree(kv->v);
        cudaFree(kv->d_page_table);
        return rc;
    }
    *out = kv.release();
    return SOC_B200_OK;
}

void soc_b200_free_kv(soc_kv* kv) {
    if (!kv) return;
    cudaSetDevice(kv->m->ctx->device);
    cudaStreamSynchronize(kv->m->ctx->stream);
    // graphs captured against this cache write its pools: a later cache may reuse the address
    if (kv->m->graph_kv == kv) {
        cudaGraphExecDestroy(kv->m->step_graph);
        kv->m->step_graph = nullptr;
        kv->m->graph_kv = nullptr;
    }
    if (kv->m->pf_graph && kv->m->pf_key.kv == kv) {
        cudaGraphExecDestroy(kv->m->pf_graph);
        kv->m->pf_graph = nullptr;
    }
    cudaFree(kv->k);
    cudaFree(kv->v);
    cudaFree(kv->d_page_table);
    delete kv;
}

int soc_b200_kv_reset(soc_kv* kv, int seq) {
    if (!kv) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        kv->check_seq(seq);
        kv->reset(seq);
    });
}

int soc_b200_kv_length(const soc_kv* kv, int seq) {
    if (!kv) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (seq < 0 || seq >= kv->max_seqs) return fail(SOC_B200_ERR_INVALID, "kv cache length batch_index out of range");
    return kv->lengths[seq];
}

int soc_b200_kv_read(soc_kv* kv, int seq, int layer, int start, int end, float* k, float* v) {
    if (!kv || !k || !v) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        soc_model* m = kv->m;
        kv->check_seq(seq);
        if (layer < 0 || static_cast<size_t>(layer) >= m->cfg.layers)
            throw Error(SOC_B200_ERR_INVALID, "kv cache read layer_index out of range");
        if (start < 0 || start > end) throw Error(SOC_B200_ERR_INVALID, "kv cache read range must be ordered");
        if (end > kv->lengths[seq]) throw Error(SOC_B200_ERR_INVALID, "kv cache read range exceeds cached sequence length");
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        const size_t hkv = m->cfg.hkv, D = m->cfg.hd, pt = kv->page_tokens;
        std::vector<uint16_t> hk(pt * hkv * D), hv(pt * hkv * D);
        const KVLayerView lv = kv->view(layer);
        for (int p = start; p < end;) {
            const int pi = p / static_cast<int>(pt);
            const int page = kv->pages[seq][pi];
            const size_t base = static_cast<size_t>(page) * hkv * pt * D;
            SOCB_CUDA(cudaMemcpy(hk.data(), lv.k + base, hk.size() * 2, cudaMemcpyDeviceToHost));
            SOCB_CUDA(cudaMemcpy(hv.data(), lv.v + base, hv.size() * 2, cudaMemcpyDeviceToHost));
            const int pend = std::min(end, (pi + 1) * static_cast<int>(pt));
            for (; p < pend; ++p) {
                const size_t slot = static_cast<size_t>(p) % pt;
                for (size_t h = 0; h < hkv; ++h)
                    for (size_t d = 0; d < D; ++d) {
                        const size_t src = (h * pt + slot) * D + d;
                        const size_t dst = (static_cast<size_t>(p - start) * hkv + h) * D + d;
                        k[dst] = half_bits_to_float(hk[src]);
                        v[dst] = half_bits_to_float(hv[src]);
                    }
            }
        }
    });
}

int soc_b200_kv_fill_random(soc_kv* kv, int seq, int n_tokens, unsigned long long seed) {
    if (!kv) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        soc_model* m = kv->m;
        kv->check_seq(seq);
        if (n_tokens < 0) throw Error(SOC_B200_ERR_INVALID, "kv fill length must not be negative");
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        cudaStream_t st = m->ctx->stream;
        kv->reset(seq);
        kv->reserve(seq, n_tokens, st);
        launch_kv_fill_random(kv->k, kv->v, kv->layer_stride(), kv->d_page_table + static_cast<size_t>(seq) * kv->max_pages,
                              kv->page_tokens, static_cast<int>(m->cfg.hkv), static_cast<int>(m->cfg_full.hkv),
                              m->tp_rank * static_cast<int>(m->cfg.hkv), static_cast<int>(m->cfg.hd),
                              static_cast<int>(m->cfg.layers), n_tokens, seq, seed, st);
        kv->lengths[seq] = n_tokens;
    });
}

int soc_b200_kv_write(soc_kv* kv, int seq, int layer, int start, int end, const float* k, const float* v) {
    if (!kv || !k || !v) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        soc_model* m = kv->m;
        kv->check_seq(seq);
        if (layer < 0 || static_cast<size_t>(layer) >= m->cfg.layers)
            throw Error(SOC_B200_ERR_INVALID, "kv cache write layer_index out of range");
        if (start < 0 || start > end) throw Error(SOC_B200_ERR_INVALID, "kv cache write range must be ordered");
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        cudaStream_t st = m->ctx->stream;
        kv->reserve(seq, end, st);
        SOCB_CUDA(cudaStreamSynchronize(st));
        const size_t hkv = m->cfg.hkv, D = m->cfg.hd, pt = kv->page_tokens;
        const KVLayerView lv = kv->view(layer);
        std::vector<uint16_t> hk(hkv * D), hv(hkv * D);
        for (int p = start; p < end; ++p) {
            const int page = kv->pages[seq][p / static_cast<int>(pt)];
            const size_t slot = static_cast<size_t>(p) % pt;
            for (size_t h = 0; h < hkv; ++h) {
                for (size_t d = 0; d < D; ++d) {
                    const size_t src = (static_cast<size_t>(p - start) * hkv + h) * D + d;
                    hk[h * D + d] = float_to_half_bits(k[src]);
                    hv[h * D + d] = float_to_half_bits(v[src]);
                }
                const size_t dst = ((static_cast<size_t>(page) * hkv + h) * pt + slot) * D;
                SOCB_CUDA(cudaMemcpy(lv.k + dst, hk.data() + h * D, D * 2, cudaMemcpyHostToDevice));
                SOCB_CUDA(cudaMemcpy(lv.v + dst, hv.data() + h * D, D * 2, cudaMemcpyHostToDevice));
            }
        }
        if (end > kv->lengths[seq]) kv->lengths[seq] = end;
    });
}

int soc_b200_prefill(soc_model* m, soc_kv* kv, int seq, const int32_t* ids, int n, float* logits_last,
                     int32_t* next_id) {
    if (!m || !kv || !ids) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (kv->m != m) return fail(SOC_B200_ERR_INVALID, "kv cache belongs to another model");
    return guarded([&] {
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        prefill_impl(m, kv, seq, ids, n, false);
        m->logits_last_rows = 1;
        cudaStream_t st = m->ctx->stream;
        if (logits_last) logits_to_host(m, 1, logits_last, st);
        int nid = 0;
        SOCB_CUDA(cudaMemcpyAsync(&nid, m->d_next, sizeof(int), cudaMemcpyDeviceToHost, st));
        check_device_error(m);
        if (next_id) *next_id = nid;
    });
}

int soc_b200_decode(soc_model* m, soc_kv* kv, int n_seqs, const int* seq_ids, const int32_t* last_ids,
                    float* logits, int32_t* next_ids) {
    if (!m || !kv || !seq_ids || !last_ids) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (kv->m != m) return fail(SOC_B200_ERR_INVALID, "kv cache belongs to another model");
    return guarded([&] {
        if (n_seqs <= 0) throw Error(SOC_B200_ERR_INVALID, "decode requires at least one sequence");
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        check_ids(m, last_ids, n_seqs);
        std::vector<char> seen(kv->max_seqs, 0);
        std::vector<int> pos(n_seqs);
        int max_vis = 0;
        for (int i = 0; i < n_seqs; ++i) {
            kv->check_seq(seq_ids[i]);
            if (seen[seq_ids[i]]) throw Error(SOC_B200_ERR_INVALID, "decode sequence ids must be distinct");
            seen[seq_ids[i]] = 1;
            if (kv->lengths[seq_ids[i]] == 0)
                throw Error(SOC_B200_ERR_INVALID, "GenerationContext decode requires a prefilled KV cache");
            pos[i] = kv->lengths[seq_ids[i]];
            max_vis = std::max(max_vis, pos[i] + 1);
        }
        cudaStream_t st = m->ctx->stream;
        for (int i = 0; i < n_seqs; ++i) kv->reserve(seq_ids[i], pos[i] + 1, st);
        if (n_seqs == 1 && m->mk_ok) {
            ensure_logits(m, 1);
            SOCB_CUDA(cudaMemcpyAsync(m->mk_ids, last_ids, sizeof(int), cudaMemcpyHostToDevice, st));
            run_mk(m, kv, seq_ids[0], pos[0], 1, m->mk_ids, m->logits);
            m->logits_last_rows = 1;
            if (logits)
                SOCB_CUDA(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->cfg.vocab, cudaMemcpyDeviceToHost, st));
            if (next_ids) SOCB_CUDA(cudaMemcpyAsync(next_ids, m->mk_ids + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
            check_device_error(m);
            kv->lengths[seq_ids[0]] = pos[0] + 1;
            return;
        }
        ensure_workspace(m, n_seqs);
        SOCB_CUDA(cudaMemcpyAsync(m->d_tokens, last_ids, sizeof(int) * n_seqs, cudaMemcpyHostToDevice, st));
        SOCB_CUDA(cudaMemcpyAsync(m->d_seq, seq_ids, sizeof(int) * n_seqs, cudaMemcpyHostToDevice, st));
        SOCB_CUDA(cudaMemcpyAsync(m->d_pos, pos.data(), sizeof(int) * n_seqs, cudaMemcpyHostToDevice, st));
        forward_rows(m, kv, n_seqs, max_vis, 0, n_seqs, 0);
        m->logits_last_rows = n_seqs;
        if (logits) logits_to_host(m, n_seqs, logits, st);
        if (next_ids) SOCB_CUDA(cudaMemcpyAsync(next_ids, m->d_next, sizeof(int) * n_seqs, cudaMemcpyDeviceToHost, st));
        check_device_error(m);
        for (int i = 0; i < n_seqs; ++i) kv->lengths[seq_ids[i]] = pos[i] + 1;
    });
}

// Device-side generation: prefill, then max_new - 1 decode steps that feed each greedy id
// back on the device (no host round trip per token).
static void generate_dev(soc_model* m, soc_kv* kv, int seq, const int32_t* prompt, int n_prompt, int max_new,
                         int32_t* d_out, bool prompt_on_device, int eos = -1) {
    kv->check_seq(seq);
    m->logits_last_rows = 0;  // the device loop does not keep the steps' logits
    if (max_new <= 0) throw Error(SOC_B200_ERR_INVALID, "generate requires max_new >= 1");
    kv->reset(seq);
    cudaStream_t st = m->ctx->stream;
    kv->reserve(seq, n_prompt + max_new - 1, st);
    prefill_impl(m, kv, seq, prompt, n_prompt, prompt_on_device);
    SOCB_CUDA(cudaMemcpyAsync(d_out, m->d_next, sizeof(int), cudaMemcpyDeviceToDevice, st));
    if (max_new > 1) decode_loop(m, kv, seq, n_prompt, max_new - 1, d_out, eos);
    kv->lengths[seq] = n_prompt + max_new - 1;
}

int soc_b200_generate(soc_model* m, soc_kv* kv, int seq, const int32_t* prompt, int n_prompt, int max_new,
                      int eos_token_id, int32_t* out_ids, int* n_out) {
    if (!m || !kv || !prompt || !out_ids) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (kv->m != m) return fail(SOC_B200_ERR_INVALID, "kv cache belongs to another model");
    return guarded([&] {
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        if (n_out) *n_out = 0;
        if (max_new == 0) {
            kv->check_seq(seq);
            kv->reset(seq);
            prefill_impl(m, kv, seq, prompt, n_prompt, false);
            check_device_error(m);
            return;
        }
        int32_t* d_out = static_cast<int32_t*>(m->dmalloc(sizeof(int32_t) * max_new));
        try {
            // ids after an eos stop are never written: clear them so the scan below is defined
            if (eos_token_id >= 0) SOCB_CUDA(cudaMemsetAsync(d_out, 0xff, sizeof(int32_t) * max_new, m->ctx->stream));
            m->loop_steps_queued = 0;
            generate_dev(m, kv, seq, prompt, n_prompt, max_new, d_out, false, eos_token_id);
            SOCB_CUDA(cudaMemcpyAsync(out_ids, d_out, sizeof(int32_t) * max_new, cudaMemcpyDeviceToHost,
                                      m->ctx->stream));
            check_device_error(m);
            if (eos_token_id >= 0 && m->loop_steps_queued > 0) {
                // the graph loop counted every step it was launched for: take off those an EOS skipped
                soc_model::LoopState fin{};
                SOCB_CUDA(cudaMemcpy(&fin, m->d_loop, sizeof(fin), cudaMemcpyDeviceToHost));
                count_launches(-static_cast<long long>(m->loop_steps_queued - fin.step) * m->graph_kernels);
            }
        } catch (...) {
            m->dfree(d_out, false);
            throw;
        }
        // no captured graph holds the output buffer (the step graph reads it through LoopState)
        m->dfree(d_out, false);
        int n = max_new;
        if (eos_token_id >= 0)
            for (int i = 0; i < max_new; ++i)
                if (out_ids[i] == eos_token_id) {
                    n = i + 1;
                    break;
                }
        // Tokens generated after an EOS were computed on the device; drop them from the cache.
        kv->lengths[seq] = n_prompt + n - 1;
        if (n_out) *n_out = n;
    });
}

int soc_b200_generate_device(soc_model* m, soc_kv* kv, int seq, const int32_t* d_prompt, int n_prompt, int max_new,
                             int32_t* d_out) {
    if (!m || !kv || !d_prompt || !d_out) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (kv->m != m) return fail(SOC_B200_ERR_INVALID, "kv cache belongs to another model");
    return guarded([&] {
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        generate_dev(m, kv, seq, d_prompt, n_prompt, max_new, d_out, true);
    });
}

int soc_b200_nccl_unique_id(void* id_out) {
    if (!id_out) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        ncclUniqueId id;
        nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
        std::memcpy(id_out, &id, sizeof(id));
    });
}

int soc_b200_nccl_comm_create(soc_ctx* ctx, int nranks, int rank, const void* id, void** comm_out) {
    if (!ctx || !id || !comm_out) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(SOC_B200_ERR_INVALID, "rank must be in [0, nranks)");
    return guarded([&] {
        SOCB_CUDA(cudaSetDevice(ctx->device));
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        ncclComm_t comm = nullptr;
        nccl_check(nccl().comm_init_rank(&comm, nranks, uid, rank), "ncclCommInitRank");
        *comm_out = comm;
    });
}

int soc_b200_nccl_comm_destroy(void* comm) {
    if (!comm) return SOC_B200_OK;
    return guarded([&] { nccl_check(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy"); });
}

int soc_b200_linear(soc_ctx* ctx, int weight_format, const void* w, const void* scales, int out_features,
                    int in_features, const float* x, int rows, float* y, void* stream) {
    if (!ctx || !w || !x || !y) return fail(SOC_B200_ERR_INVALID, "null argument");
    return guarded([&] {
        if (out_features <= 0 || in_features <= 0 || rows <= 0)
            throw Error(SOC_B200_ERR_INVALID, "linear: dimensions must be positive");
        const int f = weight_format == SOC_B200_WEIGHTS_BF16       ? WF_BF16
                      : weight_format == SOC_B200_WEIGHTS_F16      ? WF_F16
                      : weight_format == SOC_B200_WEIGHTS_INT8_G64 ? WF_I8G64
                      : weight_format == SOC_B200_WEIGHTS_INT4_G32 ? WF_I4G32
                                                                   : -1;
        if (f < 0) throw Error(SOC_B200_ERR_INVALID, "linear: weight format not supported by this build");
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
        const bool quant = f == WF_I8G64 || f == WF_I4G32;
        const bool tc = tc_rows_ok(rows, out_features, in_features, f) && in_features % 64 == 0 && tc_available();
        if (!tc) {
            launch_linear(f, w, scales, out_features, in_features, x, in_features, rows, nullptr, 0.0f, y,
                          out_features, LIN_STORE, st);
            return;
        }
        if (quant && scales == nullptr) throw Error(SOC_B200_ERR_INVALID, "linear: group-quantised weights need scales");
        // scratch: input rows hi | lo (GEMM type), then the fp16 expansion of quantised weights
        const int gf = f == WF_BF16 ? WF_BF16 : WF_F16;
        const bool split = rows <= tc_split_max_rows();
        const size_t xbytes = 2 * static_cast<size_t>(rows) * in_features;
        const size_t xoff = (xbytes + 255) / 256 * 256;
        const size_t need = 2 * xoff + (quant ? 2 * static_cast<size_t>(out_features) * in_features : 0);
        if (need > ctx->lin_scratch_bytes) {
            SOCB_CUDA(cudaStreamSynchronize(st));
            if (ctx->lin_scratch) SOCB_CUDA(cudaFree(ctx->lin_scratch));
            ctx->lin_scratch = nullptr;
            ctx->lin_scratch_bytes = 0;
            SOCB_CUDA(cudaMalloc(&ctx->lin_scratch, need));
            ctx->lin_scratch_bytes = need;
        }
        char* base = static_cast<char*>(ctx->lin_scratch);
        void *xh = base, *xl = base + xoff, *wq = base + 2 * xoff;
        const void* wsrc = w;
        if (quant) {
            launch_dequant(f, w, scales, out_features, in_features, WF_F16, wq, st);
            wsrc = wq;
        }
        CUtensorMap ta{}, tl{}, tw{};
        tc_make_map(&ta, xh, gf, rows, in_features, in_features, TC_BOX_A);
        if (split) tc_make_map(&tl, xl, gf, rows, in_features, in_features, TC_BOX_A);
        tc_make_map(&tw, wsrc, gf, out_features, in_features, in_features, TC_BOX_W);
        launch_rows_to_half(gf, x, in_features, rows, in_features, nullptr, 0.0f, xh, split ? xl : nullptr,
                            in_features, st);
        launch_gemm_tc(gf, ta, split ? &tl : nullptr, tw, rows, out_features, in_features, y, out_features, LIN_STORE,
                       false, nullptr, ctx->ws(), TC_WS_FLOATS, ctx->d_err, st);
    });
}

int soc_b200_topk(soc_model* m, int row, int k, float* top_logits, int32_t* top_token_ids) {
    if (!m || !top_logits || !top_token_ids) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (k < 1 || k > TOPK_MAX) return fail(SOC_B200_ERR_INVALID, "top-k: k must be in [1, 64]");
    return guarded([&] {
        if (row < 0 || row >= m->logits_last_rows)
            throw Error(SOC_B200_ERR_INVALID, "top-k: no logits row " + std::to_string(row) +
                                                  " from the last prefill or decode call");
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        cudaStream_t st = m->ctx->stream;
        const int V = static_cast<int>(m->cfg.vocab);
        if (!m->topk_cand) {
            m->topk_cand = static_cast<unsigned long long*>(
                m->dmalloc(sizeof(unsigned long long) * static_cast<size_t>(topk_scratch_keys(V, TOPK_MAX))));
            m->topk_vals = static_cast<float*>(m->dmalloc(sizeof(float) * TOPK_MAX));
            m->topk_ids = static_cast<int*>(m->dmalloc(sizeof(int) * TOPK_MAX));
        }
        const float* base;
        int seg_len;
        size_t seg_stride;
        if (m->tp_size == 1) {
            base = m->logits + static_cast<size_t>(row) * m->v_loc;
            seg_len = V;
            seg_stride = 0;
        } else {
            // every rank makes this call: the shards of the rows are gathered, then each rank picks
            gather_logits(m, m->logits_last_rows, st);
            base = m->logits_all + static_cast<size_t>(row) * m->v_loc;
            seg_len = m->v_loc;
            seg_stride = static_cast<size_t>(m->logits_last_rows) * m->v_loc;
        }
        launch_topk(base, V, seg_len, seg_stride, m->temperature, k, m->topk_cand, m->topk_vals, m->topk_ids, st);
        SOCB_CUDA(cudaMemcpyAsync(top_logits, m->topk_vals, sizeof(float) * k, cudaMemcpyDeviceToHost, st));
        SOCB_CUDA(cudaMemcpyAsync(top_token_ids, m->topk_ids, sizeof(int) * k, cudaMemcpyDeviceToHost, st));
        SOCB_CUDA(cudaStreamSynchronize(st));
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode step that allocates nothing (soc_b200_decode_noalloc).
//
// Some hosts cannot allocate device memory while serving: for example an
// engine that hands every byte of the GPU to its own pool at start-up, or a
// caller that must not make cudaMalloc's implicit device synchronisation on its
// latency path.  This entry point runs one batch-1 decode step through the
// persistent decode kernel with all of that kernel's scratch -- the residual and
// activation vectors (tagged words), split-K attention partials, the argmax
// slots and the logits row -- in one file-scope device array of fixed size.
// Every GPU that loads this library keeps that array (kNoAllocScratchBytes)
// until the process exits.  All calls share the array and it keeps the last
// call's contents: the argmax slots are cleared at the start of each call, and
// the tags of the vectors keep growing from call to call, so no word left by an
// earlier call is taken for this call's; calls whose GPU work overlaps (other
// streams, other threads) race.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 128;
void* g_noalloc_addr[kMaxDevices] = {};
unsigned g_noalloc_tag[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on `device` (which must be current).  The host-side
// symbol is only a stand-in, so the address comes from cudaGetSymbolAddress, once per device.
void* noalloc_scratch(int device) {
    if (device < 0 || device >= kMaxDevices) throw Error(SOC_B200_ERR_INVALID, "decode_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[device] == nullptr) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            throw Error(SOC_B200_ERR_CUDA, std::string("decode_noalloc: cudaGetSymbolAddress failed: ") +
                                               cudaGetErrorString(e));
        g_noalloc_addr[device] = ptr;
    }
    return g_noalloc_addr[device];
}

// Tag base of the next call on `device`'s array: the array starts out zeroed (a static
// device array is), and it is cleared again before the tags would wrap.
unsigned noalloc_tags(int device, int steps, int L, unsigned long long* vec, size_t vec_n, unsigned long long* part,
                      size_t part_n, cudaStream_t st) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    return mk_next_tags(&g_noalloc_tag[device], steps, L, vec, vec_n, part, part_n, st);
}
}  // namespace

extern "C" int soc_b200_decode_noalloc(soc_model* m, soc_kv* kv, int seq, int32_t last_id, float* logits,
                                       int32_t* next_id) {
    if (!m || !kv) return fail(SOC_B200_ERR_INVALID, "null argument");
    if (kv->m != m) return fail(SOC_B200_ERR_INVALID, "kv cache belongs to another model");
    return guarded([&] {
        if (m->tp_size > 1)
            throw Error(SOC_B200_ERR_INVALID, "decode_noalloc: not available for a tensor-parallel shard");
        const Config& c = m->cfg;
        SOCB_CUDA(cudaSetDevice(m->ctx->device));
        cudaStream_t st = m->ctx->stream;
        const int H = static_cast<int>(c.hidden), I = static_cast<int>(c.inter), hq = static_cast<int>(c.hq);
        const int hkv = static_cast<int>(c.hkv), D = static_cast<int>(c.hd), V = static_cast<int>(c.vocab);
        const int grid = mk_grid(m->ctx->device);
        if (!mk_supported(static_cast<int>(c.layers), H, I, hq, hkv, D, V, m->wfmt, m->efmt, grid))
            throw Error(SOC_B200_ERR_INVALID, "decode_noalloc: model shape not supported by the persistent decode kernel");
        if (!m->mk_ok || m->d_mk_layers == nullptr)
            throw Error(SOC_B200_ERR_INVALID, "decode_noalloc: the model was loaded without the persistent decode kernel");
        kv->check_seq(seq);
        check_ids(m, &last_id, 1);
        const int pos = kv->lengths[seq];
        if (pos == 0) throw Error(SOC_B200_ERR_INVALID, "GenerationContext decode requires a prefilled KV cache");
        if (pos + 1 > m->rope_len) throw Error(SOC_B200_ERR_CAPACITY, "decode position beyond the RoPE table");

        int group = 1;
        const int S = mk_att_plan(pos + 1, hq, hkv, grid, &group);
        // carve the array (256-byte aligned pieces); every check comes before any side effect
        char* base = static_cast<char*>(noalloc_scratch(m->ctx->device));
        size_t off = 0;
        auto carve = [&](size_t bytes) {
            char* q = base + off;
            off += (bytes + 255) / 256 * 256;
            return static_cast<void*>(q);
        };
        const size_t nvec = mk_vec_words(H, I, hq, hkv, D);
        const size_t npart = mk_part_words(hq, hkv, D, S);
        auto* best = static_cast<unsigned long long*>(carve(sizeof(unsigned long long) * grid));
        auto* ids = static_cast<int*>(carve(sizeof(int) * 2));
        auto* vec = static_cast<unsigned long long*>(carve(sizeof(unsigned long long) * nvec));
        auto* part = static_cast<unsigned long long*>(carve(sizeof(unsigned long long) * npart));
        auto* lg = static_cast<float*>(carve(sizeof(float) * V));
        if (off > kNoAllocScratchBytes)
            throw Error(SOC_B200_ERR_CAPACITY, "decode_noalloc: this model needs " + std::to_string(off) +
                                                   " bytes of scratch, above the static maximum of " +
                                                   std::to_string(kNoAllocScratchBytes));
        // the cache's host page allocator; no device memory is allocated (the page table exists)
        kv->reserve(seq, pos + 1, st);
        SOCB_CUDA(cudaMemsetAsync(best, 0, sizeof(unsigned long long) * grid, st));
        SOCB_CUDA(cudaMemcpyAsync(ids, &last_id, sizeof(int), cudaMemcpyHostToDevice, st));
        // tags keep growing across calls on this device's array (whatever model made them), so a
        // word left by an earlier call never carries a tag this call waits for
        const unsigned tag0 = noalloc_tags(m->ctx->device, 1, static_cast<int>(c.layers), vec, nvec, part, npart, st);
        MKParams p = mk_params(m, kv, seq, pos, 1, ids, lg, -1, S, group, vec, part, best, tag0);
        mk_launch(p, grid, st);
        count_launches(1);
        if (logits) SOCB_CUDA(cudaMemcpyAsync(logits, lg, sizeof(float) * V, cudaMemcpyDeviceToHost, st));
        int nid = 0;
        SOCB_CUDA(cudaMemcpyAsync(&nid, ids + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
        check_device_error(m);
        kv->lengths[seq] = pos + 1;
        m->logits_last_rows = 0;  // this step's logits are in the static array, not the model's
        if (next_id) *next_id = nid;
    });
}
