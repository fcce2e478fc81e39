#include "mpfx.h"

#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace miniprefix_b200 {
namespace {

// A byte source over the model file that knows its own position and the file's
// size; every short read throws the message its caller names.
class ByteSource {
public:
    explicit ByteSource(const std::string& path) : path_(path), in_(path, std::ios::binary) {
        if (!in_) throw std::runtime_error("cannot open model: " + path);
    }

    bool try_take(void* out, std::size_t n) {
        if (!in_.read(static_cast<char*>(out), static_cast<std::streamsize>(n))) return false;
        at_ += n;
        return true;
    }
    void take(void* out, std::size_t n, const char* short_read) {
        if (!try_take(out, n)) throw std::runtime_error(short_read);
    }
    template <class T>
    T scalar() {
        T v{};
        take(&v, sizeof(T), "truncated model");
        return v;
    }
    std::uint64_t position() const { return at_; }
    std::uint64_t size() const { return std::filesystem::file_size(path_); }
    bool exhausted() { return in_.peek() == std::char_traits<char>::eof(); }

private:
    std::string path_;
    std::ifstream in_;
    std::uint64_t at_ = 0;
};

// The fixed header after the magic: eight int32 shape fields, two float32
// constants and the uint32 tied flag (44 bytes, read as one block; a file that
// ends inside it is "truncated model" wherever it ends).
#pragma pack(push, 1)
struct HeaderBlock {
    std::int32_t shape[8];  // layers, hidden, intermediate, heads, kv_heads, vocabulary, context, eos
    float rms_epsilon;
    float rope_theta;
    std::uint32_t tied;
};
#pragma pack(pop)
static_assert(sizeof(HeaderBlock) == 44, "MPFX0001 header is 44 bytes after the magic");

ModelConfig parse_header(ByteSource& src) {
    char magic[8];
    if (!src.try_take(magic, sizeof magic) || std::memcmp(magic, "MPFX0001", sizeof magic) != 0)
        throw std::runtime_error("invalid model format");
    HeaderBlock h{};
    src.take(&h, sizeof h, "truncated model");
    ModelConfig c;
    c.layers = h.shape[0];
    c.hidden = h.shape[1];
    c.intermediate = h.shape[2];
    c.heads = h.shape[3];
    c.kv_heads = h.shape[4];
    c.vocabulary = h.shape[5];
    c.context = h.shape[6];
    c.eos = h.shape[7];
    c.rms_epsilon = h.rms_epsilon;
    c.rope_theta = h.rope_theta;
    if (h.tied > 1) throw std::runtime_error("invalid tied flag");
    c.tied = h.tied == 1;
    c.validate();
    return c;
}

// The tensors a configuration must contain: Llama names, 2-D linears [in][out].
struct Entry {
    int rank;
    std::array<std::int32_t, 2> dims;
    bool seen = false;
};

class Directory {
public:
    explicit Directory(const ModelConfig& c) {
        const std::int32_t H = c.hidden, I = c.intermediate, V = c.vocabulary, K = c.kv_width();
        add("model.embed_tokens.weight", {V, H});
        add("model.norm.weight", {H});
        if (!c.tied) add("lm_head.weight", {H, V});
        struct LayerTensor {
            const char* suffix;
            std::vector<std::int32_t> dims;
        };
        const LayerTensor per_layer[] = {
            {"input_layernorm.weight", {H}},       {"post_attention_layernorm.weight", {H}},
            {"self_attn.q_proj.weight", {H, H}},   {"self_attn.k_proj.weight", {H, K}},
            {"self_attn.v_proj.weight", {H, K}},   {"self_attn.o_proj.weight", {H, H}},
            {"mlp.gate_proj.weight", {H, I}},      {"mlp.up_proj.weight", {H, I}},
            {"mlp.down_proj.weight", {I, H}},
        };
        for (int layer = 0; layer < c.layers; ++layer)
            for (const auto& t : per_layer) add("model.layers." + std::to_string(layer) + "." + t.suffix, t.dims);
    }
    std::size_t size() const { return entries_.size(); }
    // The entry of `name` if it is expected and not seen yet, else null.
    Entry* claim(const std::string& name) {
        const auto it = entries_.find(name);
        if (it == entries_.end() || it->second.seen) return nullptr;
        return &it->second;
    }

private:
    void add(std::string name, const std::vector<std::int32_t>& dims) {
        Entry e{int(dims.size()), {dims[0], dims.size() > 1 ? dims[1] : 0}};
        entries_.emplace(std::move(name), e);
    }
    std::unordered_map<std::string, Entry> entries_;
};

// One directory record: name, rank and dims (checked against the directory as
// they are read), payload size (checked against the shape and the bytes left in
// the file), then the float32 payload, which must be finite.
void read_tensor(ByteSource& src, Directory& dir, std::vector<float>& payload, std::string& name) {
    const auto length = src.scalar<std::uint32_t>();
    if (length < 1 || length > 256) throw std::runtime_error("invalid tensor name");
    name.assign(length, '\0');
    src.take(name.data(), length, "truncated name");
    Entry* entry = dir.claim(name);
    if (!entry) throw std::runtime_error("unknown/duplicate tensor: " + name);
    if (src.scalar<std::uint32_t>() != std::uint32_t(entry->rank)) throw std::runtime_error("tensor rank mismatch");
    std::uint64_t elements = 1;
    for (int d = 0; d < entry->rank; ++d) {
        const auto dim = src.scalar<std::int32_t>();
        if (dim != entry->dims[std::size_t(d)]) throw std::runtime_error("tensor shape mismatch: " + name);
        elements *= std::uint64_t(dim);
    }
    const auto bytes = src.scalar<std::uint64_t>();
    const std::uint64_t here = src.position(), total = src.size();
    if (bytes != elements * sizeof(float) || here > total || bytes > total - here)
        throw std::runtime_error("invalid tensor bytes");
    payload.resize(std::size_t(elements));
    src.take(payload.data(), std::size_t(bytes), "truncated tensor");
    for (const float v : payload)
        if (!std::isfinite(v)) throw std::runtime_error("nonfinite weights");
    entry->seen = true;
}

}  // namespace

ModelConfig read_mpfx_config(const std::string& path) {
    ByteSource src(path);
    return parse_header(src);
}

ModelConfig read_mpfx(const std::string& path, const std::function<void(const MpfxTensor&)>& sink) {
    ByteSource src(path);
    const ModelConfig config = parse_header(src);
    Directory dir(config);
    if (src.scalar<std::uint32_t>() != dir.size()) throw std::runtime_error("model tensor count mismatch");
    std::vector<float> payload;
    std::string name;
    for (std::size_t i = 0; i < dir.size(); ++i) {
        read_tensor(src, dir, payload, name);
        sink(MpfxTensor{name, payload.data(), payload.size()});
    }
    if (!src.exhausted()) throw std::runtime_error("trailing model data");
    return config;
}

}  // namespace miniprefix_b200
