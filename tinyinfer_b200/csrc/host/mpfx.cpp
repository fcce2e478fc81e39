#include "mpfx.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <set>
#include <stdexcept>
#include <vector>

namespace miniprefix_b200 {
namespace {

template <class T>
T read_value(std::ifstream& file) {
    T value{};
    if (!file.read(reinterpret_cast<char*>(&value), sizeof(T))) throw std::runtime_error("truncated model");
    return value;
}

ModelConfig read_header(std::ifstream& file, const std::string& path) {
    if (!file) throw std::runtime_error("cannot open model: " + path);
    char magic[8];
    if (!file.read(magic, 8) || std::memcmp(magic, "MPFX0001", 8) != 0) throw std::runtime_error("invalid model format");
    ModelConfig c;
    int* fields[] = {&c.layers, &c.hidden, &c.intermediate, &c.heads, &c.kv_heads, &c.vocabulary, &c.context, &c.eos};
    for (int* field : fields) *field = read_value<std::int32_t>(file);
    c.rms_epsilon = read_value<float>(file);
    c.rope_theta = read_value<float>(file);
    const auto tied = read_value<std::uint32_t>(file);
    if (tied > 1) throw std::runtime_error("invalid tied flag");
    c.tied = tied != 0;
    c.validate();
    return c;
}

}  // namespace

ModelConfig read_mpfx_config(const std::string& path) {
    std::ifstream file(path, std::ios::binary);
    return read_header(file, path);
}

ModelConfig read_mpfx(const std::string& path, const std::function<void(const MpfxTensor&)>& sink) {
    std::ifstream file(path, std::ios::binary);
    const ModelConfig c = read_header(file, path);
    // expected names and shapes (model.cpp:31-41)
    std::map<std::string, std::vector<std::int32_t>> expected{{"model.embed_tokens.weight", {c.vocabulary, c.hidden}},
                                                              {"model.norm.weight", {c.hidden}}};
    if (!c.tied) expected["lm_head.weight"] = {c.hidden, c.vocabulary};
    for (int layer = 0; layer < c.layers; ++layer) {
        const std::string p = "model.layers." + std::to_string(layer) + ".";
        expected[p + "input_layernorm.weight"] = {c.hidden};
        expected[p + "post_attention_layernorm.weight"] = {c.hidden};
        expected[p + "self_attn.q_proj.weight"] = {c.hidden, c.hidden};
        expected[p + "self_attn.k_proj.weight"] = {c.hidden, c.kv_width()};
        expected[p + "self_attn.v_proj.weight"] = {c.hidden, c.kv_width()};
        expected[p + "self_attn.o_proj.weight"] = {c.hidden, c.hidden};
        expected[p + "mlp.gate_proj.weight"] = {c.hidden, c.intermediate};
        expected[p + "mlp.up_proj.weight"] = {c.hidden, c.intermediate};
        expected[p + "mlp.down_proj.weight"] = {c.intermediate, c.hidden};
    }
    const auto count = read_value<std::uint32_t>(file);
    if (count != expected.size()) throw std::runtime_error("model tensor count mismatch");
    const auto file_bytes = std::filesystem::file_size(path);
    std::set<std::string> seen;
    std::vector<float> data;
    for (std::uint32_t i = 0; i < count; ++i) {
        const auto length = read_value<std::uint32_t>(file);
        if (length < 1 || length > 256) throw std::runtime_error("invalid tensor name");
        std::string name(length, '\0');
        if (!file.read(name.data(), length)) throw std::runtime_error("truncated name");
        const auto found = expected.find(name);
        if (found == expected.end() || seen.count(name)) throw std::runtime_error("unknown/duplicate tensor: " + name);
        const auto rank = read_value<std::uint32_t>(file);
        if (rank != found->second.size()) throw std::runtime_error("tensor rank mismatch");
        std::uint64_t elements = 1;
        for (std::uint32_t d = 0; d < rank; ++d) {
            const auto dim = read_value<std::int32_t>(file);
            if (dim != found->second[d]) throw std::runtime_error("tensor shape mismatch: " + name);
            elements *= std::uint64_t(dim);
        }
        const auto bytes = read_value<std::uint64_t>(file);
        const auto offset = static_cast<std::uint64_t>(file.tellg());
        if (bytes != elements * sizeof(float) || offset > file_bytes || bytes > file_bytes - offset)
            throw std::runtime_error("invalid tensor bytes");
        data.resize(std::size_t(elements));
        if (!file.read(reinterpret_cast<char*>(data.data()), static_cast<std::streamsize>(bytes)))
            throw std::runtime_error("truncated tensor");
        for (float v : data)
            if (!std::isfinite(v)) throw std::runtime_error("nonfinite weights");
        seen.insert(name);
        sink(MpfxTensor{name, data.data(), data.size()});
    }
    if (file.peek() != std::char_traits<char>::eof()) throw std::runtime_error("trailing model data");
    return c;
}

}  // namespace miniprefix_b200
