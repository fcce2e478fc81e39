// mp_paged_attention_decode_noalloc: the paged-attention decode operator for
// callers that cannot allocate device memory.
//
// Who needs it: a host process that embeds this library inside another runtime
// which owns the GPU's memory (a serving framework with its own caching
// allocator or a fixed memory budget it accounts for up front), or code on a
// path where cudaMalloc/cudaFree are not allowed because they synchronise the
// device or fail mid-run. mp_paged_attention_decode grows its scratch with
// cudaMalloc on demand; this variant never does. Its scratch -- the slice work
// list and per-row metadata, the slice partial results, the per-(row, kv head) arrival
// counters and an error word -- lives in one file-scope __device__ array of
// fixed size (kScratchBytes below, about 5 MB), which every GPU that loads the
// library holds until the process exits.
//
// Limits: at most kMaxRows sequences per call and kMaxWork slices. When
// pages_per_split is 0 the slice length is chosen to fit kMaxWork; an explicit
// pages_per_split that needs more slices, or more sequences than kMaxRows, is
// rejected with MP_ERR_INVALID and a message, before anything is queued.
//
// Sharing: all calls on a device share the one array, which keeps the last
// call's contents. Each call clears the arrival counters and the schedule (which must start at
// zero) on its stream before the kernel; the other regions are fully written
// before they are read. Calls whose device work overlaps -- on different
// streams, or from different host threads without ordering -- race on the
// array and give wrong results.
//
// Errors: bounds and timeout bits go to the caller's device_error word when one
// is given. With device_error NULL they go to an error word inside the array,
// which mp_paged_attention_status reads and clears; each call clears it before
// its kernel, so read it before the next call on the same device.
//
// Set-up: the first call on a device, with that device current, looks up the
// array's device address with cudaGetSymbolAddress (in host code the array's
// name is only a host-side stand-in, not a device address) and keeps it for
// that device; make that first call before any stream capture begins.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "miniprefix_b200.h"

namespace {

constexpr int kMaxRows = 512;
constexpr int kMaxWork = 2048;
constexpr int kMaxDevices = 64;
constexpr size_t kPartialFloats = size_t(kMaxWork) * mpb::kHeads * (mpb::kHeadDim + 2);
// Layout (bytes): partials | metadata (4 x kMaxRows row words + 4 x kMaxWork work words) |
// counters (kMaxRows x 3 kv heads) | schedule (2 words) | error
constexpr size_t kPartialBytes = kPartialFloats * sizeof(float);
constexpr size_t kMetaWords = 4 * size_t(kMaxRows) + 5 * size_t(kMaxWork);  // rows | work | order
constexpr size_t kMetaOffset = kPartialBytes;
constexpr size_t kCounterOffset = kMetaOffset + kMetaWords * sizeof(int32_t);
constexpr size_t kSchedOffset = kCounterOffset + size_t(kMaxRows) * mpb::kKvHeads * sizeof(unsigned);
constexpr size_t kErrorOffset = kSchedOffset + 2 * sizeof(unsigned);
constexpr size_t kScratchBytes = (kErrorOffset + sizeof(unsigned) + 255) / 256 * 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mutex;
unsigned char* g_scratch_address[kMaxDevices] = {};

// Host staging of the metadata: a fixed host array, so the call allocates no
// host memory either. The H2D copy reads pageable memory, which CUDA stages
// before cudaMemcpyAsync returns, so the array may be refilled by the next call.
int32_t g_host_meta[kMetaWords];

}  // namespace

extern "C" int mp_paged_attention_decode_noalloc(const float* q, const float* keys, const float* values,
                                                 int32_t layers, int32_t layer, int32_t block_tokens,
                                                 int32_t max_blocks, const int32_t* tables, int32_t table_stride,
                                                 const int32_t* lengths, int32_t count, float* out,
                                                 int32_t pages_per_split, void* stream_ptr, uint32_t* device_error) {
    if (!q || !keys || !values || !tables || !lengths || !out || count < 1 || layers < 1 || layer < 0 ||
        layer >= layers || block_tokens < 1 || max_blocks < 1 || table_stride < 1 || pages_per_split < 0) {
        mpb::set_last_error("invalid argument");
        return MP_ERR_INVALID;
    }
    if (count > kMaxRows) {
        mpb::set_last_error("mp_paged_attention_decode_noalloc: more than 512 sequences in one call");
        return MP_ERR_INVALID;
    }
    long long total_pages = 0;
    for (int i = 0; i < count; ++i) {
        if (lengths[i] < 1 || int64_t(lengths[i]) > int64_t(table_stride) * block_tokens) {
            mpb::set_last_error("sequence length outside its block table");
            return MP_ERR_INVALID;
        }
        total_pages += (lengths[i] + block_tokens - 1) / block_tokens;
    }
    // Slices. pages_per_split 0: one equal run of pages per CTA
    // (mpb::plan_static_runs: at most kMaxRows + kAttnPersistentCtas items, which
    // fits kMaxWork); else slices of that many pages, pulled longest first.
    auto slices = [&](int pps) {
        long long n = 0;
        for (int i = 0; i < count; ++i) n += std::max(1, ((lengths[i] + block_tokens - 1) / block_tokens + pps - 1) / pps);
        return n;
    };
    static_assert(kMaxRows + mpb::kAttnPersistentCtas <= kMaxWork, "static runs fit the work list");
    const int pps = pages_per_split;
    if (pps != 0 && slices(pps) > kMaxWork) {
        mpb::set_last_error("mp_paged_attention_decode_noalloc: more than 2048 slices; raise pages_per_split");
        return MP_ERR_INVALID;
    }
    (void)total_pages;

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
        mpb::set_last_error("no usable current CUDA device");
        return MP_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
        void* address = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&address, g_noalloc_scratch);
        if (e != cudaSuccess || !address) {
            mpb::set_last_error(cudaGetErrorString(e));
            return MP_ERR_CUDA;
        }
        g_scratch_address[device] = static_cast<unsigned char*>(address);
    }
    unsigned char* base = g_scratch_address[device];
    float* partial = reinterpret_cast<float*>(base);
    int32_t* meta = reinterpret_cast<int32_t*>(base + kMetaOffset);
    unsigned* counters = reinterpret_cast<unsigned*>(base + kCounterOffset);
    unsigned* sched = reinterpret_cast<unsigned*>(base + kSchedOffset);
    unsigned* error = reinterpret_cast<unsigned*>(base + kErrorOffset);

    // Row arrays (slot, length, slices, first slice) then the work list.
    int work = 0;
    int32_t* rows = g_host_meta;
    int32_t* items = g_host_meta + 4 * count;
    auto pages_of = [&](int r) { return (lengths[r] + block_tokens - 1) / block_tokens; };
    auto emit = [&](int r, int b, int e, int k) {
        if (k == 0) rows[3 * count + r] = work;
        rows[2 * count + r] = k + 1;
        items[4 * work] = r;
        items[4 * work + 1] = b;
        items[4 * work + 2] = e;
        items[4 * work + 3] = k;
        ++work;
    };
    for (int r = 0; r < count; ++r) {
        rows[r] = r;
        rows[count + r] = lengths[r];
    }
    int runs = 0;
    int32_t* order = nullptr;  // after the work list: the longest-first order, or the runs' first items
    if (pps == 0) {
        // the runs' first items follow the work list, whose final length is only
        // known at the end: collect them at the top of the order region's maximum
        // extent, then move them down
        int32_t* starts = g_host_meta + 4 * count + 4 * kMaxWork;
        starts[0] = 0;
        runs = mpb::plan_static_runs(count, pages_of, emit, [&](int c, int it) { starts[c] = it; });
        order = items + 4 * work;
        std::memmove(order, starts, size_t(runs + 1) * sizeof(int32_t));
    } else {
        for (int r = 0; r < count; ++r) {
            const int n = std::max(1, (pages_of(r) + pps - 1) / pps);
            for (int k = 0; k < n; ++k) emit(r, k * pps, std::min(pages_of(r), (k + 1) * pps), k);
        }
        order = items + 4 * work;
    }
    // processing order of the persistent kernel: longest slices first (insertion
    // sort into the fixed array; at most kMaxWork items)
    for (int i = 0; i < (runs ? 0 : work); ++i) {
        auto tokens = [&](int k) {
            return std::min(items[4 * k + 2] * block_tokens, int(lengths[items[4 * k]])) - items[4 * k + 1] * block_tokens;
        };
        const int ti = tokens(i);
        int j = i;
        while (j > 0 && tokens(order[j - 1]) < ti) {
            order[j] = order[j - 1];
            --j;
        }
        order[j] = i;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const size_t tail = runs ? size_t(runs) + 1 : size_t(work);
    cudaError_t e = cudaMemcpyAsync(meta, g_host_meta, (size_t(4 * count + 4 * work) + tail) * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(counters, 0, size_t(count) * mpb::kKvHeads * sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(sched, 0, 2 * sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(error, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = mpb::configure_attention();
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
    p.row_slot = meta;
    p.row_len = meta + count;
    p.row_splits = meta + 2 * count;
    p.row_work0 = meta + 3 * count;
    p.work = reinterpret_cast<const mpb::AttnWork*>(meta + 4 * count);
    p.work_count = work;
    p.order = runs ? nullptr : meta + 4 * count + 4 * work;
    p.cta_items = runs ? meta + 4 * count + 4 * work : nullptr;
    p.cta_count = runs;
    p.partial = partial;
    p.counters = counters;
    p.sched = sched;
    p.out = out;
    p.out_stride = mpb::kQWidth;
    p.error = device_error ? reinterpret_cast<unsigned*>(device_error) : error;
    e = mpb::launch_paged_attention(p, stream);
    if (e != cudaSuccess) {
        mpb::set_last_error(cudaGetErrorString(e));
        return MP_ERR_CUDA;
    }
    return MP_OK;
}

cudaError_t mpb::noalloc_take_error(cudaStream_t stream, unsigned* bits) {
    *bits = 0;
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        base = g_scratch_address[device];
    }
    if (!base) return cudaSuccess;  // no call on this device yet
    unsigned* error = reinterpret_cast<unsigned*>(base + kErrorOffset);
    unsigned word = 0;
    e = cudaMemcpyAsync(&word, error, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && word) e = cudaMemsetAsync(error, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) *bits = word;
    return e;
}
