#include "b200_runner.h"

#include <algorithm>
#include <cmath>
#include <exception>

namespace miniprefix_b200 {
namespace {

void device_check(int rc, const char* what) {
    if (rc != MP_OK) throw std::runtime_error(std::string(what) + ": " + mp_last_error());
}

mp_model_config to_device(const ModelConfig& c) {
    mp_model_config m{};
    m.layers = c.layers;
    m.hidden = c.hidden;
    m.intermediate = c.intermediate;
    m.heads = c.heads;
    m.kv_heads = c.kv_heads;
    m.vocabulary = c.vocabulary;
    m.context = c.context;
    m.eos = c.eos;
    m.rms_epsilon = c.rms_epsilon;
    m.rope_theta = c.rope_theta;
    m.tied = c.tied ? 1 : 0;
    return m;
}

}  // namespace

B200Runner::B200Runner(const ModelConfig& config, int context, KvCacheConfig kv, B200Options options)
    : config_(config), kv_(kv, config.layers, config.kv_width(), context, config.vocabulary), options_(options) {
    if (context < 1 || context > config.context) throw std::invalid_argument("invalid runner context");
    const int bt = kv.block_tokens;
    table_stride_ = (config.context + bt - 1) / bt;
    mp_runtime_config rt{};
    rt.block_tokens = bt;
    rt.max_blocks = kv.max_blocks;
    rt.max_sequences = options.max_sequences;
    rt.table_stride = table_stride_;
    rt.max_step_tokens = options.max_step_tokens;
    rt.max_step_sequences = options.max_step_sequences;
    const mp_model_config m = to_device(config);
    device_check(mp_create(options.device, &m, &rt, &ctx_), "create B200 context");
    for (int s = options.max_sequences - 1; s >= 0; --s) free_slots_.push_back(s);
    mirror_.assign(std::size_t(options.max_sequences), {});
    written_epoch_.assign(std::size_t(kv.max_blocks), 0);
    read_epoch_.assign(std::size_t(kv.max_blocks), 0);
    pending_epoch_.assign(std::size_t(options.max_sequences), 0);
    const std::size_t kvw = std::size_t(config.kv_width());
    stats_.device_workspace_bytes =
        std::size_t(options.max_step_tokens) *
        (std::size_t(config.hidden) * 5 + kvw * 2 + std::size_t(config.intermediate)) * sizeof(float);
    stats_.device_allocations = 1;
}

B200Runner::~B200Runner() {
    drain();
    if (ctx_) mp_destroy(ctx_);
}

void B200Runner::drain() noexcept {
    if (ctx_) mp_sync(ctx_, options_.timeout_ms);
}

void B200Runner::set_weight(const std::string& name, const float* data, std::size_t elements) {
    device_check(mp_set_weight(ctx_, name.c_str(), data, elements), "upload weight");
    stats_.weight_uploaded_bytes += elements * sizeof(float);
    stats_.device_weight_bytes += elements * sizeof(float);
}

void B200Runner::finalize_weights() { device_check(mp_finalize_weights(ctx_), "finalize weights"); }

int B200Runner::slot_of(const RequestId& id) const { return slots_.at(id); }

void B200Runner::create(const RequestId& id) {
    if (kv_.contains(id)) throw std::invalid_argument("sequence already exists");
    if (free_slots_.empty()) throw std::runtime_error("no free device block-table slot");
    kv_.create(id);
    const int slot = free_slots_.back();
    free_slots_.pop_back();
    slots_[id] = slot;
    mirror_[std::size_t(slot)].clear();
    if (checkpoint_) checkpoint_->created.emplace_back(id, slot);
}

void B200Runner::free_slot(const RequestId& id) {
    auto it = slots_.find(id);
    if (it == slots_.end()) return;
    const int slot = it->second;
    slots_.erase(it);
    mirror_[std::size_t(slot)].clear();
    if (checkpoint_) checkpoint_->released.emplace_back(id, slot);
    // Queued device work may still read this slot's table.
    if (descs_.empty()) free_slots_.push_back(slot);
    else quarantine_.push_back(slot);
}

void B200Runner::fork_sequence(const RequestId& source, const RequestId& target) {
    flush();
    kv_.fork_sequence(source, target);
    mirror_[std::size_t(slot_of(target))].clear();  // uploaded with the next append
}

void B200Runner::mark_pending_reads(const RequestId& id) {
    if (descs_.empty() || !kv_.contains(id)) return;
    const auto it = slots_.find(id);
    if (it == slots_.end() || pending_epoch_[std::size_t(it->second)] != epoch_) return;
    for (int b : kv_.sequence(id).blocks) read_epoch_[std::size_t(b)] = epoch_;
}

std::size_t B200Runner::reuse_prefix(const RequestId& id, const std::vector<TokenId>& prompt) {
    mark_pending_reads(id);
    const std::size_t used = kv_.reuse_prefix(id, prompt);
    mirror_[std::size_t(slot_of(id))].clear();  // the table goes up with the next append
    return used;
}

void B200Runner::clear_prefix_cache() {
    flush();
    drain();
    kv_.clear_prefix_cache();
}

// Entries of `sequence.blocks` that differ from what the device already holds,
// looking from index `from` on (entries before it are known to be in sync).
void B200Runner::table_entries(int slot, const PagedSequence& sequence, std::vector<mp_table_entry>& out,
                               std::size_t from) {
    auto& m = mirror_[std::size_t(slot)];
    const auto& b = sequence.blocks;
    if (m.size() < from) from = 0;  // the mirror was dropped: compare everything
    if (m.size() < b.size()) m.resize(b.size(), -1);
    for (std::size_t i = from; i < b.size(); ++i)
        if (m[i] != b[i]) {
            out.push_back({slot, int32_t(i), b[i]});
            m[i] = b[i];
        }
}

std::vector<float> B200Runner::append(const RequestId& id, const std::vector<TokenId>& tokens) {
    flush();
    auto tx = kv_.prepare_append(id, tokens);
    const auto& sequence = tx.sequence();
    const int slot = slot_of(id);
    if (tx.tail_copy()) ++costs_.cow_pages;
    std::vector<mp_tail_copy_region> regions;
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) {
        regions.push_back({r.destination, r.source, r.pitch, r.width, r.rows});
        costs_.cow_bytes += 2 * r.width * r.rows * sizeof(float);
    });
    std::vector<mp_table_entry> entries;
    table_entries(slot, sequence, entries);
    std::vector<float> logits(std::size_t(config_.vocabulary));
    int32_t token = 0, finite = 0;
    mp_cow_timing(ctx_, cost_timing_ && !regions.empty());
    // A forward carries at most max_step_tokens tokens: longer appends run as
    // consecutive forwards of the same sequence (the table entries and the copy
    // with the first); only the last returns logits, as only the last row's are
    // the append's result.
    const int n = int(tokens.size()), step = std::max(options_.max_step_tokens, 1);
    int rc = MP_OK;
    for (int off = 0; off < n && (rc == MP_OK || rc == MP_ERR_NONFINITE); off += step) {
        const bool first = off == 0, last = off + step >= n;
        const mp_sequence_desc desc{slot, sequence.used + off, std::min(step, n - off)};
        rc = mp_forward(ctx_, &desc, 1, tokens.data() + off, first ? entries.data() : nullptr,
                        first ? int32_t(entries.size()) : 0, first ? regions.data() : nullptr,
                        first ? int32_t(regions.size()) : 0, &token, &finite, last ? logits.data() : nullptr,
                        options_.timeout_ms);
        if (!last && rc == MP_ERR_NONFINITE) rc = MP_OK;  // only the final row's logits count
        if (first && cost_timing_ && !regions.empty() && rc != MP_ERR_CUDA && rc != MP_ERR_TIMEOUT) {
            float ms = 0.f;
            mp_cow_elapsed(ctx_, &ms);
            costs_.cow_copy_ns += std::uint64_t(double(ms) * 1e6);
            ++costs_.cow_timed_copies;
        }
    }
    stats_.token_uploaded_bytes += tokens.size() * sizeof(TokenId);
    stats_.block_table_uploaded_bytes += entries.size() * sizeof(int32_t);
    if (rc != MP_OK) {
        mirror_[std::size_t(slot)].clear();  // re-upload the whole table next time
        if (rc == MP_ERR_NONFINITE) throw std::runtime_error("nonfinite CUDA logits");
        throw std::runtime_error(std::string("B200 forward: ") + mp_last_error());
    }
    for (float v : logits)
        if (!std::isfinite(v)) throw std::runtime_error("nonfinite CUDA logits");
    tx.commit();
    stats_.logits_downloaded_bytes += logits.size() * sizeof(float);
    return logits;
}

void B200Runner::begin_batch() {
    results_.clear();
    kv_.begin_checkpoint();
    checkpoint_ = std::make_unique<Checkpoint>();
    checkpoint_->stats = stats_;
    checkpoint_->costs = costs_;
}

std::size_t B200Runner::stage_append(const RequestId& id, const std::vector<TokenId>& tokens) {
    auto tx = kv_.prepare_append(id, tokens);
    const auto& sequence = tx.sequence();
    const int slot = slot_of(id);
    const std::size_t ticket = results_.size();
    results_.push_back({});
    const auto& copy = tx.tail_copy();
    if (!replay_ && int(tokens.size()) > options_.max_step_tokens)
        throw std::invalid_argument("append larger than the runner's max_step_tokens");
    if (!replay_ && !descs_.empty()) {
        // Capacity of one device forward.
        if (int(descs_.size()) + 1 > options_.max_step_sequences ||
            tokens_.size() + tokens.size() > std::size_t(options_.max_step_tokens))
            flush();
    }
    if (!replay_ && !descs_.empty()) {
        // The device applies a step as: every COW source read, then every COW
        // destination written, then per layer every new K/V row written before any
        // attention reads. Sequential order differs from that only when (1) a COW
        // source was written by an earlier pending append, (2) this append writes a
        // page (COW destination or new page) that an earlier pending append's
        // attention still reads -- a page freed this step by that sequence -- or
        // (3) the sequence already has a pending append. A page freed this step that
        // pending work only read as a COW source is safe to reuse.
        auto reused = [&](int b) {
            return kv_.freed_this_epoch(b) && read_epoch_[std::size_t(b)] == epoch_;
        };
        bool hazard = pending_epoch_[std::size_t(slot)] == epoch_;
        if (copy && written_epoch_[std::size_t(copy->source)] == epoch_) hazard = true;
        if (copy && reused(copy->destination)) hazard = true;
        for (std::size_t b = tx.original_blocks(); b < sequence.blocks.size() && !hazard; ++b)
            hazard = reused(sequence.blocks[b]);
        if (hazard) {
            ++hazard_flushes_;
            flush();
        }
    }
    if (copy) ++costs_.cow_pages;
    const std::size_t region_start = regions_.size();
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) {
        regions_.push_back({r.destination, r.source, r.pitch, r.width, r.rows});
        costs_.cow_bytes += 2 * r.width * r.rows * sizeof(float);
    });
    if (replay_) {
        regions_.resize(region_start);
        mirror_[std::size_t(slot)].clear();
        tx.commit();
        return ticket;
    }
    // an append changes at most its last original page (copy on write) and the
    // pages after it; the mirror is dropped whenever anything else may change
    table_entries(slot, sequence, entries_, tx.original_blocks() ? tx.original_blocks() - 1 : 0);
    const int bt = kv_.config().block_tokens;
    for (int p = sequence.used / bt; p <= (sequence.used + int(tokens.size()) - 1) / bt; ++p)
        written_epoch_[std::size_t(sequence.blocks[std::size_t(p)])] = epoch_;
    pending_epoch_[std::size_t(slot)] = epoch_;
    descs_.push_back({slot, sequence.used, int32_t(tokens.size())});
    tokens_.insert(tokens_.end(), tokens.begin(), tokens.end());
    tickets_.push_back(ticket);
    if (capture_) pending_ids_.push_back(id);
    tx.commit();
    return ticket;
}

void B200Runner::set_logits_capture(bool on) {
    if (!descs_.empty()) flush();
    capture_ = on;
    pending_ids_.clear();
    if (!on) captured_.clear();
}

bool B200Runner::captured_logits(const RequestId& id, std::vector<float>& out) const {
    const auto it = captured_.find(id);
    if (it == captured_.end()) return false;
    out = it->second;
    return true;
}

void B200Runner::flush() {
    if (descs_.empty()) {
        kv_.settle_publishes();
        kv_.next_epoch();
        ++epoch_;
        return;
    }
    const int n = int(descs_.size());
    out_tokens_.assign(std::size_t(n), 0);
    out_finite_.assign(std::size_t(n), 0);
    const bool timed = cost_timing_ && !regions_.empty();
    mp_cow_timing(ctx_, timed);
    // mp_forward in three parts: the step's queued prefix-cache publishes run on
    // the host between the launch and the wait for the device.
    int rc = mp_forward_prepare(ctx_, descs_.data(), n, tokens_.data(), entries_.data(), int32_t(entries_.size()),
                                regions_.data(), int32_t(regions_.size()));
    std::string error;
    std::exception_ptr publish_error;
    if (rc == MP_OK) {
        rc = mp_forward_launch(ctx_);
        if (rc == MP_OK) {
            try {
                kv_.settle_publishes();
            } catch (...) {
                publish_error = std::current_exception();
            }
        } else {
            error = mp_last_error();
        }
        // after a failed launch this still waits for what was enqueued and ends the step
        const std::size_t vocabulary = std::size_t(config_.vocabulary);
        if (capture_) out_logits_.assign(std::size_t(n) * vocabulary, 0.f);
        const int collected = mp_forward_collect(ctx_, out_tokens_.data(), out_finite_.data(),
                                                 capture_ ? out_logits_.data() : nullptr, options_.timeout_ms);
        if (capture_ && collected == MP_OK && pending_ids_.size() == std::size_t(n)) {
            for (int i = 0; i < n; ++i)
                captured_[pending_ids_[std::size_t(i)]].assign(out_logits_.begin() + std::ptrdiff_t(i * vocabulary),
                                                               out_logits_.begin() + std::ptrdiff_t((i + 1) * vocabulary));
            stats_.logits_downloaded_bytes += out_logits_.size() * sizeof(float);
        }
        if (rc == MP_OK) rc = collected;
    }
    if (rc != MP_OK && error.empty()) error = mp_last_error();
    ++flushes_;
    stats_.token_uploaded_bytes += tokens_.size() * sizeof(TokenId);
    stats_.block_table_uploaded_bytes += entries_.size() * sizeof(int32_t);
    if ((rc != MP_OK && rc != MP_ERR_NONFINITE) || publish_error) {
        for (auto& m : mirror_) m.clear();
        descs_.clear();
        tokens_.clear();
        entries_.clear();
        regions_.clear();
        tickets_.clear();
    pending_ids_.clear();
        if (publish_error) std::rethrow_exception(publish_error);
        throw std::runtime_error(std::string("B200 forward: ") + error);
    }
    if (timed) {
        float ms = 0.f;
        mp_cow_elapsed(ctx_, &ms);
        costs_.cow_copy_ns += std::uint64_t(double(ms) * 1e6);
        costs_.cow_timed_copies += regions_.size();
    }
    for (int i = 0; i < n; ++i) {
        auto& r = results_[tickets_[std::size_t(i)]];
        r.token = out_tokens_[std::size_t(i)];
        r.finite = out_finite_[std::size_t(i)] != 0;
    }
    descs_.clear();
    tokens_.clear();
    entries_.clear();
    regions_.clear();
    tickets_.clear();
    pending_ids_.clear();
    for (int s : quarantine_) free_slots_.push_back(s);
    quarantine_.clear();
    kv_.next_epoch();
    ++epoch_;
}

void B200Runner::restore_batch() {
    if (!checkpoint_) throw std::logic_error("no runner checkpoint");
    descs_.clear();
    tokens_.clear();
    entries_.clear();
    regions_.clear();
    tickets_.clear();
    pending_ids_.clear();
    kv_.restore_checkpoint();
    // Undo slot moves newest first, then forget every device-table mirror.
    auto& cp = *checkpoint_;
    for (auto it = cp.released.rbegin(); it != cp.released.rend(); ++it) {
        auto q = std::find(quarantine_.begin(), quarantine_.end(), it->second);
        if (q != quarantine_.end()) quarantine_.erase(q);
        auto f = std::find(free_slots_.begin(), free_slots_.end(), it->second);
        if (f != free_slots_.end()) free_slots_.erase(f);
        slots_[it->first] = it->second;
    }
    for (auto it = cp.created.rbegin(); it != cp.created.rend(); ++it) {
        slots_.erase(it->first);
        free_slots_.push_back(it->second);
    }
    for (auto& m : mirror_) m.clear();
    stats_ = cp.stats;
    costs_ = cp.costs;
    checkpoint_.reset();
    results_.clear();
}

void B200Runner::fail_append(const RequestId& id, const std::vector<TokenId>& tokens) {
    auto tx = kv_.prepare_append(id, tokens);
    if (tx.tail_copy()) ++costs_.cow_pages;
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) {
        costs_.cow_bytes += 2 * r.width * r.rows * sizeof(float);
    });
    mirror_[std::size_t(slot_of(id))].clear();
    throw std::runtime_error("nonfinite CUDA logits");  // tx rolls back on unwinding
}

void B200Runner::end_batch() {
    flush();
    kv_.end_checkpoint();
    checkpoint_.reset();
    results_.clear();
}

void B200Runner::release(const RequestId& id) {
    mark_pending_reads(id);
    kv_.release(id);
    free_slot(id);
}

void B200Runner::clear() {
    descs_.clear();
    tokens_.clear();
    entries_.clear();
    regions_.clear();
    tickets_.clear();
    pending_ids_.clear();
    const int rc = ctx_ ? mp_sync(ctx_, options_.timeout_ms) : MP_OK;
    kv_.end_checkpoint();
    checkpoint_.reset();
    kv_.clear();
    for (const auto& [id, slot] : slots_) free_slots_.push_back(slot);
    for (int s : quarantine_) free_slots_.push_back(s);
    quarantine_.clear();
    slots_.clear();
    for (auto& m : mirror_) m.clear();
    if (rc != MP_OK && rc != MP_ERR_BOUNDS) throw std::runtime_error(std::string("clear completion: ") + mp_last_error());
}

RunnerStats B200Runner::stats() const {
    RunnerStats r = stats_;
    r.update_kv_stats(kv_.stats());
    r.block_table_device_bytes = slots_.size() * std::size_t(table_stride_) * sizeof(int32_t);
    return r;
}

CostStats B200Runner::cost_stats() const {
    CostStats r = kv_.cost_stats();
    r.cow_pages = costs_.cow_pages;
    r.cow_bytes = costs_.cow_bytes;
    r.cow_copy_ns = costs_.cow_copy_ns;
    r.cow_timed_copies = costs_.cow_timed_copies;
    return r;
}

void B200Runner::set_cost_timing(bool enabled) {
    cost_timing_ = enabled;
    kv_.set_cost_timing(enabled);
}

void RunnerStats::update_kv_stats(const KvStats& s) {
    live_sequences = s.live_sequences;
    live_kv_bytes = s.live_kv_bytes;
    peak_kv_bytes = s.peak_kv_bytes;
    forward_tokens = s.forward_tokens;
    kv_block_tokens = s.kv_block_tokens;
    kv_total_blocks = s.kv_total_blocks;
    kv_live_blocks = s.kv_live_blocks;
    kv_peak_blocks = s.kv_peak_blocks;
    kv_reserved_bytes = s.kv_reserved_bytes;
    prefix_cache_capacity = s.prefix_cache_capacity;
    kv_cached_blocks = s.kv_cached_blocks;
    kv_cache_only_blocks = s.kv_cache_only_blocks;
    prefix_hits = s.prefix_hits;
    prefix_misses = s.prefix_misses;
    prefix_reused_tokens = s.prefix_reused_tokens;
    prefix_evictions = s.prefix_evictions;
}

void ModelConfig::validate() const {
    if (layers < 1 || layers > 128 || hidden < 2 || hidden > 8192 || intermediate < 1 || intermediate > 65536 ||
        heads < 1 || kv_heads < 1 || hidden % heads || heads % kv_heads || (hidden / heads) % 2 ||
        hidden / heads > 256 || vocabulary < 2 || vocabulary > 262144 || context < 1 || context > 131072 || eos < 0 ||
        eos >= vocabulary || !std::isfinite(rms_epsilon) || rms_epsilon <= 0 || !std::isfinite(rope_theta) ||
        rope_theta <= 1)
        throw std::invalid_argument("unsupported/invalid Llama configuration");
}

std::size_t ModelRunner::stage_append(const RequestId& id, const std::vector<TokenId>& tokens) {
    const auto logits = append(id, tokens);
    AppendResult r;
    r.finite = true;
    for (float v : logits) r.finite = r.finite && std::isfinite(v);
    r.token = TokenId(std::max_element(logits.begin(), logits.end()) - logits.begin());
    results_.push_back(r);
    return results_.size() - 1;
}

}  // namespace miniprefix_b200
