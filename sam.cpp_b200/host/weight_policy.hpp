// weight_policy.hpp -- which GGUF type every SAM 3 image tensor must have, and
// the checks a loader runs on a checkpoint's quantization metadata before it
// uploads any weight.  Host-side C++17 on top of gguf_reader.hpp (no GGML).
//
// Mirrors the weight-precision policy of the reference loader (paths relative
// to the SAM.cpp tree, src/models/sam3/weights.hpp):
//   image_profile / modular_profile      <- image_quantization_profile,
//                                           modular_image_quantization_profile (:64-94)
//   parse_modules / modules_match_profile <- parse_image_quantization_modules,
//                                           image_quantization_modules_match_profile (:96-134)
//   image_tensor_type                    <- image_quantized_tensor_type (:136-177), including the
//                                           Q8_0 fallback of the 4736-wide vision fc2 rows (:154-164)
//   modular_linear_weight / modular_tensor_type
//                                        <- image_modular_linear_weight,
//                                           image_modular_quantized_tensor_type (:179-248)
//   parse_mixed_policy / mixed_tensor_type / read_mixed_policy
//                                        <- parse_image_mixed_policy (:250-312),
//                                           image_mixed_quantized_tensor_type (:314-341),
//                                           read_image_mixed_policy (:343-369)
//   inspect_weight_policy                <- the precision part of inspect_weights (:496-620):
//                                           schema 1-7, storage profile, file type, quantization
//                                           version, the fixed SAM 3 image parameters and global
//                                           block order, the 1133-tensor count, and the expected type
//                                           of every tensor.  The tokenizer asset checks of
//                                           inspect_weights belong to text tokenization, not to
//                                           weight precision, and are not repeated here.
// The mixed policy's identity is the SHA-256 of its canonical text (FIPS 180-4,
// sha256_hex below).  Error texts follow the reference's where a caller may
// match on them.
#pragma once

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "gguf_reader.hpp"

namespace sam::internal::samq_policy {

using samq_io::GgufReader;
using samq_io::GgufTensor;
using samq_io::GgufValueType;

// GGML type ids (ggml_type) of the storage types the policy assigns.
enum : int { kF32 = 0, kF16 = 1, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14 };

inline int block_size(int type) { return type == kQ8_0 ? 32 : (type == kQ4_K || type == kQ5_K || type == kQ6_K) ? 256 : 1; }

// ---- SHA-256 (FIPS 180-4) ---------------------------------------------------

inline std::string sha256_hex(const std::string& message) {
    static constexpr std::uint32_t k[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
        0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
        0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
        0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
        0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
        0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
        0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
        0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
    std::uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                          0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    auto rotr = [](std::uint32_t x, int n) { return (x >> n) | (x << (32 - n)); };
    std::vector<std::uint8_t> data(message.begin(), message.end());
    const std::uint64_t bit_length = static_cast<std::uint64_t>(message.size()) * 8;
    data.push_back(0x80);
    while (data.size() % 64 != 56) data.push_back(0);
    for (int i = 7; i >= 0; --i) data.push_back(static_cast<std::uint8_t>(bit_length >> (8 * i)));
    for (std::size_t chunk = 0; chunk < data.size(); chunk += 64) {
        std::uint32_t w[64];
        for (int i = 0; i < 16; ++i)
            w[i] = (std::uint32_t(data[chunk + 4 * i]) << 24) | (std::uint32_t(data[chunk + 4 * i + 1]) << 16) |
                   (std::uint32_t(data[chunk + 4 * i + 2]) << 8) | std::uint32_t(data[chunk + 4 * i + 3]);
        for (int i = 16; i < 64; ++i) {
            const std::uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const std::uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        std::uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; ++i) {
            const std::uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
            const std::uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
    static const char* hex = "0123456789abcdef";
    std::string out;
    for (std::uint32_t v : h)
        for (int i = 7; i >= 0; --i) out.push_back(hex[(v >> (4 * i)) & 15]);
    return out;
}

// ---- profiles --------------------------------------------------------------

// Schema-3 profiles: quantize the ViT linears (and, for image-linear-*, the
// text encoder's).
struct ImageProfile {
    const char* name;
    const char* precision;
    int type;
    std::uint32_t file_type;
    bool quantize_text_linear;
};

inline const ImageProfile* image_profile(const std::string& name) {
    static constexpr std::array<ImageProfile, 8> profiles{{
        {"image-linear-q8_0-v1", "q8_0", kQ8_0, 7, true},
        {"image-linear-q6_k-v1", "q6_k", kQ6_K, 18, true},
        {"image-linear-q5_k-v1", "q5_k", kQ5_K, 16, true},
        {"image-linear-q4_k-v1", "q4_k", kQ4_K, 14, true},
        {"image-vision-linear-q8_0-v1", "q8_0", kQ8_0, 7, false},
        {"image-vision-linear-q6_k-v1", "q6_k", kQ6_K, 18, false},
        {"image-vision-linear-q5_k-v1", "q5_k", kQ5_K, 16, false},
        {"image-vision-linear-q4_k-v1", "q4_k", kQ4_K, 14, false},
    }};
    for (const auto& p : profiles)
        if (name == p.name) return &p;
    return nullptr;
}

// Schema-4 profiles: quantize the linears of a list of modules (full presets
// require all four modules).
struct ModularProfile {
    const char* name;
    const char* precision;
    int type;
    std::uint32_t file_type;
    bool full_preset;
};

inline const ModularProfile* modular_profile(const std::string& name) {
    static constexpr std::array<ModularProfile, 8> profiles{{
        {"image-full-linear-q8_0-v1", "q8_0", kQ8_0, 7, true},
        {"image-full-linear-q6_k-v1", "q6_k", kQ6_K, 18, true},
        {"image-full-linear-q5_k-v1", "q5_k", kQ5_K, 16, true},
        {"image-full-linear-q4_k-v1", "q4_k", kQ4_K, 14, true},
        {"image-modules-linear-q8_0-v1", "q8_0", kQ8_0, 7, false},
        {"image-modules-linear-q6_k-v1", "q6_k", kQ6_K, 18, false},
        {"image-modules-linear-q5_k-v1", "q5_k", kQ5_K, 16, false},
        {"image-modules-linear-q4_k-v1", "q4_k", kQ4_K, 14, false},
    }};
    for (const auto& p : profiles)
        if (name == p.name) return &p;
    return nullptr;
}

inline const std::array<const char*, 4>& module_order() {
    static constexpr std::array<const char*, 4> modules{{"vision", "text", "fusion", "decoder"}};
    return modules;
}

// A nonempty, strictly canonical-order subset of vision,text,fusion,decoder.
inline std::vector<std::string> parse_modules(const std::string& csv) {
    if (csv.empty()) throw std::runtime_error("schema-4 quantization module list is empty");
    std::vector<std::string> result;
    int previous = -1;
    std::size_t begin = 0;
    for (;;) {
        const std::size_t comma = csv.find(',', begin);
        const std::string token = csv.substr(begin, comma == std::string::npos ? std::string::npos : comma - begin);
        int index = -1;
        for (std::size_t i = 0; i < module_order().size(); ++i)
            if (token == module_order()[i]) index = static_cast<int>(i);
        if (index <= previous)
            throw std::runtime_error("schema-4 quantization modules must be a nonempty canonical CSV list");
        previous = index;
        result.push_back(token);
        if (comma == std::string::npos) break;
        begin = comma + 1;
    }
    return result;
}

inline bool modules_match_profile(const ModularProfile& profile, const std::vector<std::string>& modules) {
    if (modules.empty()) return false;
    if (!profile.full_preset) return true;
    if (modules.size() != module_order().size()) return false;
    for (std::size_t i = 0; i < modules.size(); ++i)
        if (modules[i] != module_order()[i]) return false;
    return true;
}

// ---- which tensors are linears of which module -------------------------------

// `name` is "<prefix><layer>.<suffix>" for some layer < layers.
inline bool indexed_layer_weight(const std::string& name, const std::string& prefix, int layers,
                                 std::initializer_list<const char*> suffixes) {
    if (name.compare(0, prefix.size(), prefix) != 0) return false;
    for (int layer = 0; layer < layers; ++layer) {
        const std::string lp = prefix + std::to_string(layer) + ".";
        if (name.compare(0, lp.size(), lp) != 0) continue;
        for (const char* s : suffixes)
            if (name.size() == lp.size() + std::strlen(s) && name.compare(lp.size(), std::string::npos, s) == 0)
                return true;
    }
    return false;
}

inline bool is_vision_linear(const std::string& name) {
    return indexed_layer_weight(name, "vit.blocks.", 32,
                                {"attn.qkv.weight", "attn.proj.weight", "mlp.lin1.weight", "mlp.lin2.weight"});
}

inline bool is_text_block_linear(const std::string& name) {
    return indexed_layer_weight(name, "text.blocks.", 24,
                                {"attn.in_proj.weight", "attn.out_proj.weight", "mlp.fc1.weight", "mlp.fc2.weight"});
}

// The 4736-wide vision fc2 rows, stored as Q8_0 by every K-quant profile.
inline bool is_fc2_fallback(const std::string& name) {
    return indexed_layer_weight(name, "vit.blocks.", 32, {"mlp.lin2.weight"});
}

inline bool modular_linear_weight(const std::string& name, const std::string& module) {
    if (module == "vision") return is_vision_linear(name);
    if (module == "text") return name == "text.resizer.weight" || is_text_block_linear(name);
    if (module == "fusion")
        return indexed_layer_weight(name, "fenc.layers.", 6,
                                    {"sa.in_proj_weight", "sa.out_proj.weight", "ca.in_proj_weight",
                                     "ca.out_proj.weight", "linear1.weight", "linear2.weight"});
    if (module != "decoder") return false;
    if (indexed_layer_weight(name, "ddec.layers.", 6,
                             {"sa.in_proj_weight", "sa.out_proj.weight", "ca.in_proj_weight", "ca.out_proj.weight",
                              "ca_text.in_proj_weight", "ca_text.out_proj.weight", "linear1.weight",
                              "linear2.weight"}))
        return true;
    if (indexed_layer_weight(name, "geom.layers.", 3,
                             {"sa.in_proj_weight", "sa.out_proj.weight", "ca.in_proj_weight", "ca.out_proj.weight",
                              "linear1.weight", "linear2.weight"}))
        return true;
    for (const char* head : {"ddec.bbox_embed.layers.", "ddec.presence_token_head.layers.",
                             "seg.mask_predictor.mask_embed.layers."})
        if (indexed_layer_weight(name, head, 3, {"weight"})) return true;
    if (indexed_layer_weight(name, "ddec.ref_point_head.layers.", 2, {"weight"})) return true;
    for (const char* axis : {"ddec.boxRPB_embed_x.layers.", "ddec.boxRPB_embed_y.layers."})
        if (indexed_layer_weight(name, axis, 2, {"weight"})) return true;
    for (const char* fixed : {"scoring.prompt_proj.weight", "scoring.hs_proj.weight", "scoring.prompt_mlp.layers.0.weight",
                              "scoring.prompt_mlp.layers.1.weight", "geom.points_direct_project.weight",
                              "geom.boxes_direct_project.weight", "geom.boxes_pos_enc_project.weight",
                              "geom.points_pool_project.weight", "geom.points_pos_enc_project.weight",
                              "geom.final_proj.weight", "seg.cross_attend_prompt.in_proj_weight",
                              "seg.cross_attend_prompt.out_proj.weight"})
        if (name == fixed) return true;
    return false;
}

// ---- expected types ------------------------------------------------------------

// Schema 3.  dimensions[0] is the row width.
inline int image_tensor_type(const std::string& name, const std::vector<std::int64_t>& dimensions,
                             const ImageProfile& profile) {
    const bool eligible = is_vision_linear(name) || (profile.quantize_text_linear && is_text_block_linear(name));
    if (!eligible) return kF32;
    const int block = block_size(profile.type);
    if (block == 256 && !dimensions.empty() && dimensions[0] == 4736 && is_fc2_fallback(name)) return kQ8_0;
    if (block == 256 && (dimensions.empty() || dimensions[0] % block != 0))
        throw std::runtime_error("K quantization profile has a noncanonical row width: " + name);
    return profile.type;
}

// Schema 4 (and the building block of the mixed policy).
inline int modular_tensor_type(const std::string& name, const std::vector<std::int64_t>& dimensions,
                               const ModularProfile& profile, const std::vector<std::string>& modules) {
    if (dimensions.size() != 2) return kF32;
    bool eligible = false;
    for (const char* module : module_order())
        eligible = eligible || (std::find(modules.begin(), modules.end(), module) != modules.end() &&
                                modular_linear_weight(name, module));
    if (!eligible) return kF32;
    const std::int64_t width = dimensions[0];
    if (width <= 0 || width % 32 != 0) return kF32;
    if (profile.type == kQ8_0 || width % 256 == 0) return profile.type;
    if (width == 4736 && is_fc2_fallback(name)) return kQ8_0;
    return kF32;
}

// ---- mixed (schema 5/6/7) policy -------------------------------------------------

struct MixedPolicy {
    std::string base_precision, policy_sha256, storage_profile;
    std::vector<std::pair<std::string, std::string>> module_precisions;  // canonical module order
    std::vector<std::pair<std::string, std::string>> tensor_precisions;  // sorted exact-name overrides
};

inline bool quantized_format(const std::string& value) {
    return modular_profile("image-full-linear-" + value + "-v1") != nullptr;
}

inline bool policy_name_char(char c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' || c == '.';
}

// Parses and authenticates a mixed allocation: the canonical text
//   "sam3:<storage profile>\nbase=<base>\n<module>=<format>\n x4 [tensor:<name>=<format>\n ...]"
// must hash (SHA-256, lowercase hex) to policy_sha256.
inline MixedPolicy parse_mixed_policy(const std::string& base_precision, const std::string& csv,
                                      const std::string& policy_sha256, const std::string& tensor_csv = "",
                                      const std::string& storage_profile = "") {
    if (!quantized_format(base_precision)) throw std::runtime_error("invalid mixed SAM base precision");
    if (csv.size() > 256) throw std::runtime_error("mixed SAM module precision CSV exceeds its bound");
    MixedPolicy result;
    result.base_precision = base_precision;
    result.policy_sha256 = policy_sha256;
    const std::string default_profile = tensor_csv.empty() ? "image-mixed-linear-v1" : "image-tensor-mixed-linear-v1";
    result.storage_profile = storage_profile.empty() ? default_profile : storage_profile;
    const bool allow_f16 = result.storage_profile == "image-mixed-f16-linear-v1";
    if (!allow_f16 && result.storage_profile != default_profile)
        throw std::runtime_error("mixed SAM profile does not match its policy version");
    auto valid_value = [&](const std::string& v) { return v == "f32" || (allow_f16 && v == "f16") || quantized_format(v); };
    bool requested_f16 = false;
    std::string encoded = "sam3:" + result.storage_profile + "\nbase=" + base_precision + "\n";
    std::size_t begin = 0;
    for (const char* module : module_order()) {
        if (begin > csv.size()) throw std::runtime_error("mixed SAM module precisions require all four modules");
        const std::size_t comma = csv.find(',', begin);
        const std::string token = csv.substr(begin, comma == std::string::npos ? std::string::npos : comma - begin);
        const std::string prefix = std::string(module) + "=";
        const std::string value = token.size() >= prefix.size() ? token.substr(prefix.size()) : "";
        if (token.compare(0, prefix.size(), prefix) != 0 || !valid_value(value))
            throw std::runtime_error("mixed SAM module precisions must be canonical module=format CSV");
        result.module_precisions.emplace_back(module, value);
        requested_f16 = requested_f16 || value == "f16";
        encoded += std::string(module) + "=" + value + "\n";
        begin = comma == std::string::npos ? csv.size() + 1 : comma + 1;
    }
    if (begin != csv.size() + 1) throw std::runtime_error("mixed SAM module precision CSV has extra entries");
    if (tensor_csv.size() > 65536) throw std::runtime_error("tensor precision CSV exceeds its bound");
    begin = 0;
    while (!tensor_csv.empty() && begin <= tensor_csv.size()) {
        const std::size_t comma = tensor_csv.find(',', begin);
        const std::string field =
            tensor_csv.substr(begin, comma == std::string::npos ? std::string::npos : comma - begin);
        const std::size_t equal = field.find('=');
        const std::string name = field.substr(0, equal);
        const std::string value = equal == std::string::npos ? "" : field.substr(equal + 1);
        if (name.empty() || name.size() > 127 || !std::all_of(name.begin(), name.end(), policy_name_char) ||
            !valid_value(value) ||
            (!result.tensor_precisions.empty() && name <= result.tensor_precisions.back().first) ||
            result.tensor_precisions.size() >= 348)
            throw std::runtime_error("invalid, duplicate or unsorted exact tensor precision override");
        bool eligible = false;
        for (const char* module : module_order()) eligible = eligible || modular_linear_weight(name, module);
        if (!eligible) throw std::runtime_error("tensor override is not a SAM linear weight: " + name);
        result.tensor_precisions.emplace_back(name, value);
        requested_f16 = requested_f16 || value == "f16";
        encoded += "tensor:" + name + "=" + value + "\n";
        if (comma == std::string::npos) break;
        begin = comma + 1;
    }
    if (allow_f16 && !requested_f16) throw std::runtime_error("mixed F16 policy must explicitly request F16");
    if (sha256_hex(encoded) != policy_sha256)
        throw std::runtime_error("mixed SAM policy SHA-256 does not match its allocation");
    return result;
}

inline int mixed_tensor_type(const std::string& name, const std::vector<std::int64_t>& dimensions,
                             const MixedPolicy& policy) {
    const std::vector<std::string> all(module_order().begin(), module_order().end());
    const ModularProfile& q8 = *modular_profile("image-full-linear-q8_0-v1");
    for (const auto& entry : policy.tensor_precisions) {
        if (entry.first != name) continue;
        if (modular_tensor_type(name, dimensions, q8, all) == kF32)
            throw std::runtime_error("tensor override targets protected/ineligible storage: " + name);
        if (entry.second == "f32") return kF32;
        if (entry.second == "f16" && policy.storage_profile == "image-mixed-f16-linear-v1") return kF16;
        const ModularProfile* profile = modular_profile("image-full-linear-" + entry.second + "-v1");
        if (!profile) throw std::runtime_error("invalid resolved tensor precision");
        return modular_tensor_type(name, dimensions, *profile, all);
    }
    for (const auto& entry : policy.module_precisions) {
        if (entry.second == "f32" || !modular_linear_weight(name, entry.first)) continue;
        if (entry.second == "f16" && policy.storage_profile == "image-mixed-f16-linear-v1")
            return modular_tensor_type(name, dimensions, q8, {entry.first}) == kF32 ? kF32 : kF16;
        const ModularProfile* profile = modular_profile("image-full-linear-" + entry.second + "-v1");
        if (!profile) throw std::runtime_error("invalid resolved mixed SAM module precision");
        return modular_tensor_type(name, dimensions, *profile, {entry.first});
    }
    return kF32;
}

inline bool has_key(const GgufReader& reader, const std::string& key) { return reader.metadata().count(key) != 0; }

inline MixedPolicy read_mixed_policy(const GgufReader& reader) {
    const std::uint32_t schema = reader.u32("sam.schema_version");
    const std::string storage_profile = reader.string("sam.storage_profile");
    const char* expected = schema == 5 ? "image-mixed-linear-v1"
                           : schema == 6 ? "image-tensor-mixed-linear-v1"
                                         : "image-mixed-f16-linear-v1";
    if ((schema != 5 && schema != 6 && schema != 7) || storage_profile != expected)
        throw std::runtime_error("mixed SAM weights require the matching schema-5/6/7 profile");
    if (has_key(reader, "sam.quantization.modules"))
        throw std::runtime_error("mixed SAM weights require module formats instead of a module list");
    std::string tensor_csv;
    if (schema == 6 || (schema == 7 && has_key(reader, "sam.quantization.tensor_precisions"))) {
        tensor_csv = reader.string("sam.quantization.tensor_precisions", 65536);
    } else if (has_key(reader, "sam.quantization.tensor_precisions")) {
        throw std::runtime_error("tensor override metadata requires schema 6/7");
    }
    MixedPolicy policy = parse_mixed_policy(reader.string("sam.quantization.base_precision", 8),
                                            reader.string("sam.quantization.module_precisions", 256),
                                            reader.string("sam.quantization.policy_sha256", 64), tensor_csv,
                                            storage_profile);
    for (const auto& entry : policy.tensor_precisions) {
        const auto& tensors = reader.tensors();
        const auto found = std::find_if(tensors.begin(), tensors.end(),
                                        [&](const GgufTensor& t) { return t.name == entry.first; });
        if (found == tensors.end()) throw std::runtime_error("unused exact tensor override: " + entry.first);
        (void)mixed_tensor_type(found->name, found->dimensions, policy);
    }
    const ModularProfile* base = modular_profile("image-full-linear-" + policy.base_precision + "-v1");
    if (reader.u32("general.file_type") != base->file_type)
        throw std::runtime_error("SAM GGUF file type does not match its mixed base precision");
    if (reader.u32("general.quantization_version") != 2)
        throw std::runtime_error("unsupported GGML quantization version");
    return policy;
}

// ---- the checkpoint-level check ----------------------------------------------

// F32 / F16 checkpoints: tensors the F16 export keeps in F32.
inline bool tensor_kept_f32(const std::string& name, std::size_t rank) {
    if (rank == 1) return true;
    for (const char* part : {"embed", "tpos", "pe_gaussian", "token", "no_obj", "no_mem", "gamma", "freqs_cis"})
        if (name.find(part) != std::string::npos) return true;
    return false;
}

struct WeightPolicy {
    std::uint32_t schema = 0;
    std::uint32_t file_type = 0;
    bool quantized = false, modular = false, mixed = false;
    std::string precision, storage_profile;
    std::vector<std::string> quantization_modules;
    const ImageProfile* image = nullptr;
    const ModularProfile* modular_profile = nullptr;
    MixedPolicy mixed_policy;

    // The GGUF type a tensor of this checkpoint must be stored as.
    int expected_type(const std::string& name, const std::vector<std::int64_t>& dimensions) const {
        if (mixed) return mixed_tensor_type(name, dimensions, mixed_policy);
        if (modular) return modular_tensor_type(name, dimensions, *modular_profile, quantization_modules);
        if (quantized) return image_tensor_type(name, dimensions, *image);
        return file_type == 1 && !tensor_kept_f32(name, dimensions.size()) ? kF16 : kF32;
    }
};

inline const std::array<std::pair<const char*, std::uint32_t>, 22>& sam3_image_parameters() {
    static const std::array<std::pair<const char*, std::uint32_t>, 22> parameters{{
        {"sam3.vision.image_size", 1008}, {"sam3.vision.patch_size", 14}, {"sam3.vision.embedding_length", 1024},
        {"sam3.vision.block_count", 32}, {"sam3.vision.attention.head_count", 16},
        {"sam3.vision.feed_forward_length", 4736}, {"sam3.vision.window_size", 24},
        {"sam3.text.embedding_length", 1024}, {"sam3.text.attention.head_count", 16}, {"sam3.text.block_count", 24},
        {"sam3.text.context_length", 32}, {"sam3.text.vocab_size", 49408}, {"sam3.text.output_length", 256},
        {"sam3.neck.embedding_length", 256}, {"sam3.fusion.block_count", 6}, {"sam3.fusion.attention.head_count", 8},
        {"sam3.fusion.feed_forward_length", 2048}, {"sam3.decoder.block_count", 6},
        {"sam3.decoder.attention.head_count", 8}, {"sam3.decoder.feed_forward_length", 2048},
        {"sam3.decoder.query_count", 200}, {"sam3.geometry.block_count", 3}}};
    return parameters;
}

// The precision checks of the reference's inspect_weights for a text-image
// checkpoint; throws std::runtime_error on the first violation.
// `expected_tensors` is 1133 for a complete SAM 3 image checkpoint; 0 skips the
// count (partial files, tests).
inline WeightPolicy inspect_weight_policy(const GgufReader& reader, std::size_t expected_tensors = 1133) {
    WeightPolicy result;
    auto require_string = [&](const char* key, const char* expected) {
        if (reader.string(key) != expected) throw std::runtime_error(std::string("unsupported SAM GGUF metadata: ") + key);
    };
    require_string("general.architecture", "sam3");
    result.schema = reader.u32("sam.schema_version");
    if (result.schema < 1 || result.schema > 7) throw std::runtime_error("unsupported SAM GGUF schema version");
    if (result.schema == 2) throw std::runtime_error("video SAM checkpoints are not image checkpoints");
    result.quantized = result.schema >= 3;
    result.modular = result.schema == 4;
    result.mixed = result.schema >= 5;
    for (const char* key : {"sam.quantization.base_precision", "sam.quantization.module_precisions",
                            "sam.quantization.policy_sha256"})
        if (!result.mixed && has_key(reader, key))
            throw std::runtime_error("mixed SAM weight metadata requires schema 5/6/7");
    if (result.schema != 6 && result.schema != 7 && has_key(reader, "sam.quantization.tensor_precisions"))
        throw std::runtime_error("tensor override metadata requires schema 6/7");
    if (result.quantized && !has_key(reader, "sam.storage_profile"))
        throw std::runtime_error("quantized SAM GGUF is missing its storage profile");
    require_string("sam.task", "text_image");
    result.file_type = reader.u32("general.file_type");
    if (result.quantized) {
        result.storage_profile = reader.string("sam.storage_profile");
        if (result.mixed) {
            result.mixed_policy = read_mixed_policy(reader);
            result.precision = "mixed";
            for (const auto& entry : result.mixed_policy.module_precisions) {
                bool selected = entry.second != "f32" && entry.second != "f16";
                for (const auto& t : result.mixed_policy.tensor_precisions)
                    selected = selected || (t.second != "f32" && t.second != "f16" &&
                                            modular_linear_weight(t.first, entry.first));
                if (selected) result.quantization_modules.push_back(entry.first);
            }
        } else if (result.modular) {
            result.modular_profile = modular_profile(result.storage_profile);
            if (!result.modular_profile) throw std::runtime_error("unsupported modular SAM GGUF quantization profile");
            result.quantization_modules = parse_modules(reader.string("sam.quantization.modules", 64));
            if (!modules_match_profile(*result.modular_profile, result.quantization_modules))
                throw std::runtime_error("SAM modular profile does not match its canonical module list");
            if (result.file_type != result.modular_profile->file_type)
                throw std::runtime_error("SAM GGUF file type does not match its modular profile");
            result.precision = result.modular_profile->precision;
        } else {
            result.image = image_profile(result.storage_profile);
            if (!result.image) throw std::runtime_error("unsupported SAM GGUF quantization profile");
            if (result.file_type != result.image->file_type)
                throw std::runtime_error("SAM GGUF file type does not match its quantization profile");
            result.precision = result.image->precision;
        }
        if (reader.u32("general.quantization_version") != 2)
            throw std::runtime_error("unsupported GGML quantization version");
    } else {
        if (result.file_type > 1) throw std::runtime_error("SAM GGUF precision must be F32 or mixed F16");
        if (has_key(reader, "sam.storage_profile")) throw std::runtime_error("unsupported SAM GGUF storage profile");
        result.precision = result.file_type == 0 ? "f32" : "f16";
    }
    for (const auto& parameter : sam3_image_parameters())
        if (reader.u32(parameter.first) != parameter.second)
            throw std::runtime_error(std::string("unsupported SAM 3 image parameter: ") + parameter.first);
    const auto& globals = reader.array("sam3.vision.global_attention_blocks", GgufValueType::Uint32, 4);
    std::array<std::uint32_t, 4> indices{};
    std::memcpy(indices.data(), globals.raw.data(), sizeof(indices));
    if (indices != std::array<std::uint32_t, 4>{7, 15, 23, 31})
        throw std::runtime_error("unsupported SAM 3 global attention block order");
    if (expected_tensors && reader.tensors().size() != expected_tensors)
        throw std::runtime_error("SAM 3 GGUF tensor count does not match its task profile");
    for (const auto& tensor : reader.tensors()) {
        if (!std::all_of(tensor.name.begin(), tensor.name.end(), policy_name_char))
            throw std::runtime_error("invalid SAM 3 tensor name: " + tensor.name);
        if (tensor.type != result.expected_type(tensor.name, tensor.dimensions))
            throw std::runtime_error("incompatible SAM 3 tensor precision: " + tensor.name);
    }
    return result;
}

}  // namespace sam::internal::samq_policy
