// mp_paged_attention_decode: the paged-attention decode operator on caller
// buffers (one query row per sequence), with an internal per-device scratch
// (work list, per-row metadata, slice partials, arrival counters) that grows on
// demand.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.h"
#include "miniprefix_b200.h"

namespace {

struct Scratch {
    int32_t* meta = nullptr;  // row arrays + work list
    size_t meta_capacity = 0;
    float* partial = nullptr;
    size_t partial_capacity = 0;  // work items
    unsigned* counters = nullptr;
    size_t counter_capacity = 0;
    unsigned* error = nullptr;
    unsigned* sched = nullptr;  // [2] persistent schedule of the decode kernel (zero between launches)
};

std::mutex g_scratch_mutex;
Scratch g_scratch[64];

template <class T>
cudaError_t grow(T*& p, size_t& capacity, size_t need, cudaStream_t stream, bool zero) {
    if (need <= capacity) return cudaSuccess;
    cudaError_t e = cudaStreamSynchronize(stream);  // in-flight launches may still use the old buffer
    if (e != cudaSuccess) return e;
    if (p) cudaFree(p);
    p = nullptr;
    capacity = 0;
    need = std::max(need, size_t(1024));
    e = cudaMalloc(reinterpret_cast<void**>(&p), need * sizeof(T));
    if (e != cudaSuccess) return e;
    if (zero) {
        e = cudaMemsetAsync(p, 0, need * sizeof(T), stream);
        if (e != cudaSuccess) return e;
    }
    capacity = need;
    return cudaSuccess;
}

}  // namespace

extern "C" int mp_paged_attention_decode(const float* q, const float* keys, const float* values, int32_t layers,
                                         int32_t layer, int32_t block_tokens, int32_t max_blocks,
                                         const int32_t* tables, int32_t table_stride, const int32_t* lengths,
                                         int32_t count, float* out, int32_t pages_per_split, void* stream_ptr) {
    if (!q || !keys || !values || !tables || !lengths || !out || count < 1 || layers < 1 || layer < 0 ||
        layer >= layers || block_tokens < 1 || max_blocks < 1 || table_stride < 1) {
        mpb::set_last_error("invalid argument");
        return MP_ERR_INVALID;
    }
    for (int i = 0; i < count; ++i)
        if (lengths[i] < 1 || int64_t(lengths[i]) > int64_t(table_stride) * block_tokens) {
            mpb::set_last_error("sequence length outside its block table");
            return MP_ERR_INVALID;
        }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return MP_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    Scratch& s = g_scratch[device];
    // Work list. pages_per_split 0: the rows' pages cut into one equal run per CTA
    // (mpb::plan_static_runs; `order` then holds the runs' first items); else
    // slices of that many pages pulled longest first by a persistent wave.
    std::vector<int32_t> host(size_t(count) * 4);
    std::vector<mpb::AttnWork> work;
    std::vector<int32_t> order;
    int runs = 0;
    auto pages_of = [&](int r) { return (lengths[r] + block_tokens - 1) / block_tokens; };
    for (int r = 0; r < count; ++r) {
        host[r] = r;              // slot
        host[count + r] = lengths[r];  // length
    }
    if (pages_per_split <= 0) {
        order.push_back(0);
        runs = mpb::plan_static_runs(
            count, pages_of,
            [&](int r, int b, int e, int k) {
                if (k == 0) host[3 * count + r] = int(work.size());  // first work item
                host[2 * count + r] = k + 1;                         // splits
                work.push_back({r, b, e, k});
            },
            [&](int, int items) { order.push_back(items); });
    } else {
        const int pps = pages_per_split;
        for (int r = 0; r < count; ++r) {
            const int n = std::max(1, (pages_of(r) + pps - 1) / pps);
            host[2 * count + r] = n;                 // splits
            host[3 * count + r] = int(work.size());  // first work item
            for (int k = 0; k < n; ++k) work.push_back({r, k * pps, std::min(pages_of(r), (k + 1) * pps), k});
        }
        // processing order of the persistent kernel: longest slices first
        order.resize(work.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = int32_t(i);
        auto tokens = [&](int32_t i) {
            const auto& w = work[i];
            return std::min(w.page_end * block_tokens, int(lengths[w.row])) - w.page_begin * block_tokens;
        };
        std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return tokens(a) > tokens(b); });
    }
    const size_t words = host.size() + 4 * work.size() + order.size();
    cudaError_t e = grow(s.meta, s.meta_capacity, words, stream, false);
    if (e == cudaSuccess) e = grow(s.partial, s.partial_capacity, work.size() * mpb::kHeads * (mpb::kHeadDim + 2),
                                   stream, false);
    if (e == cudaSuccess) e = grow(s.counters, s.counter_capacity, size_t(count) * mpb::kKvHeads, stream, true);
    if (e == cudaSuccess && !s.sched) {
        e = cudaMalloc(reinterpret_cast<void**>(&s.sched), 2 * sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemsetAsync(s.sched, 0, 2 * sizeof(unsigned), stream);
    }
    if (e == cudaSuccess && !s.error) {
        e = cudaMalloc(reinterpret_cast<void**>(&s.error), sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemsetAsync(s.error, 0, sizeof(unsigned), stream);
    }
    if (e == cudaSuccess) e = mpb::configure_attention();
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? MP_ERR_NOMEM : MP_ERR_CUDA;
    }
    host.resize(words);
    std::copy(reinterpret_cast<const int32_t*>(work.data()), reinterpret_cast<const int32_t*>(work.data()) + 4 * work.size(),
              host.begin() + 4 * count);
    std::copy(order.begin(), order.end(), host.begin() + 4 * count + 4 * work.size());
    // Pageable source: the copy is staged before cudaMemcpyAsync returns.
    e = cudaMemcpyAsync(s.meta, host.data(), words * 4, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return MP_ERR_CUDA;
    }
    mpb::AttnParams p{};
    p.q = q;
    p.q_stride = mpb::kQWidth;
    p.keys = keys;
    p.values = values;
    p.page_stride = layers;  // caller pools: the reference layout [block][layer][slot][192]
    p.layer_offset = layer;
    p.block_tokens = block_tokens;
    p.max_blocks = max_blocks;
    p.tables = tables;
    p.table_stride = table_stride;
    p.row_slot = s.meta;
    p.row_len = s.meta + count;
    p.row_splits = s.meta + 2 * count;
    p.row_work0 = s.meta + 3 * count;
    p.work = reinterpret_cast<const mpb::AttnWork*>(s.meta + 4 * count);
    p.work_count = int(work.size());
    const int32_t* tail = s.meta + 4 * count + 4 * work.size();  // order, or the runs' first items
    p.order = runs ? nullptr : tail;
    p.cta_items = runs ? tail : nullptr;
    p.cta_count = runs;
    p.partial = s.partial;
    p.counters = s.counters;
    p.sched = s.sched;
    p.out = out;
    p.out_stride = mpb::kQWidth;
    p.error = s.error;
    e = mpb::launch_paged_attention(p, stream);
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return MP_ERR_CUDA;
    }
    return MP_OK;
}

extern "C" int mp_paged_attention_prefill(const float* q, const float* keys, const float* values, int32_t layers,
                                          int32_t layer, int32_t block_tokens, int32_t max_blocks,
                                          const int32_t* tables, int32_t table_stride, const int32_t* seq_starts,
                                          const int32_t* seq_counts, int32_t count, float* out, void* stream_ptr) {
    if (!q || !keys || !values || !tables || !seq_starts || !seq_counts || !out || count < 1 || layers < 1 ||
        layer < 0 || layer >= layers || block_tokens < 1 || max_blocks < 1 || table_stride < 1) {
        mpb::set_last_error("invalid argument");
        return MP_ERR_INVALID;
    }
    // Tiles of up to kPrefillTileRows rows per (sequence, kv head), the longest
    // context first (the planner of the forward does the same).
    std::vector<mpb::PrefillWork> work;
    int row = 0;
    for (int i = 0; i < count; ++i) {
        if (seq_starts[i] < 0 || seq_counts[i] < 1 ||
            int64_t(seq_starts[i]) + seq_counts[i] > int64_t(table_stride) * block_tokens) {
            mpb::set_last_error("sequence rows outside its block table");
            return MP_ERR_INVALID;
        }
        for (int t = 0; t * mpb::kPrefillTileRows < seq_counts[i]; ++t)
            for (int kh = 0; kh < mpb::kKvHeads; ++kh)
                work.push_back({row + t * mpb::kPrefillTileRows,
                                std::min(mpb::kPrefillTileRows, seq_counts[i] - t * mpb::kPrefillTileRows),
                                seq_starts[i] + t * mpb::kPrefillTileRows, i, kh, {0, 0, 0}});
        row += seq_counts[i];
    }
    std::stable_sort(work.begin(), work.end(), [](const mpb::PrefillWork& a, const mpb::PrefillWork& b) {
        return a.position + a.rows > b.position + b.rows;
    });
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return MP_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    Scratch& s = g_scratch[device];
    const size_t words = work.size() * sizeof(mpb::PrefillWork) / sizeof(int32_t);
    cudaError_t e = grow(s.meta, s.meta_capacity, words, stream, false);
    if (e == cudaSuccess && !s.error) {
        e = cudaMalloc(reinterpret_cast<void**>(&s.error), sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemsetAsync(s.error, 0, sizeof(unsigned), stream);
    }
    if (e == cudaSuccess) e = mpb::configure_prefill_attention();
    // pageable source: staged before cudaMemcpyAsync returns
    if (e == cudaSuccess) e = cudaMemcpyAsync(s.meta, work.data(), words * 4, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? MP_ERR_NOMEM : MP_ERR_CUDA;
    }
    mpb::PrefillParams p{};
    p.q = q;
    p.q_stride = mpb::kQWidth;
    p.keys = keys;
    p.values = values;
    p.page_stride = layers;  // caller pools: the reference layout [block][layer][slot][192]
    p.layer_offset = layer;
    p.block_tokens = block_tokens;
    p.max_blocks = max_blocks;
    p.tables = tables;
    p.table_stride = table_stride;
    p.work = reinterpret_cast<const mpb::PrefillWork*>(s.meta);
    p.work_count = int(work.size());
    p.out = out;
    p.out_stride = mpb::kQWidth;
    p.error = s.error;
    e = mpb::launch_prefill_attention(p, stream);
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return MP_ERR_CUDA;
    }
    return MP_OK;
}

// Reads and clears the operators' device error words on the current device
// (synchronises `stream`): the allocating operator's, and the word that
// mp_paged_attention_decode_noalloc writes when its caller passes no
// device_error. Returns MP_OK, MP_ERR_BOUNDS or MP_ERR_TIMEOUT. After a timeout
// the arrival counters and the schedule of the allocating operator are cleared:
// a CTA that gave up never counted its slice, and leftover counts would make the
// next call merge at the wrong slice.
extern "C" int mp_paged_attention_status(void* stream_ptr) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return MP_ERR_CUDA;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    unsigned err = 0;
    if (mpb::noalloc_take_error(stream, &err) != cudaSuccess) return MP_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    Scratch& s = g_scratch[device];
    if (s.error) {
        unsigned own = 0;
        if (cudaMemcpyAsync(&own, s.error, sizeof(unsigned), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            return MP_ERR_CUDA;
        if (own) {
            if (cudaMemsetAsync(s.error, 0, sizeof(unsigned), stream) != cudaSuccess) return MP_ERR_CUDA;
            if (own & mpb::kErrTimeout) {
                if (cudaMemsetAsync(s.counters, 0, s.counter_capacity * sizeof(unsigned), stream) != cudaSuccess ||
                    cudaMemsetAsync(s.sched, 0, 2 * sizeof(unsigned), stream) != cudaSuccess)
                    return MP_ERR_CUDA;
            }
        }
        err |= own;
    }
    if (!err) return MP_OK;
    return (err & mpb::kErrTimeout) ? MP_ERR_TIMEOUT : MP_ERR_BOUNDS;
}
