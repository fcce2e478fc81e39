#include "engine.h"

#include <algorithm>
#include <cmath>
#include <map>
#include <set>

namespace miniprefix_b200 {
namespace {

SchedulerConfig scheduler_config(const EngineConfig& config) {
    if (config.max_batch_size < 1 || config.token_budget < 1 || config.prefill_chunk < 1)
        throw std::invalid_argument("invalid engine configuration");
    return {config.max_batch_size, config.token_budget, config.prefill_chunk};
}

}  // namespace

Engine::Engine(std::unique_ptr<ModelRunner> runner, EngineConfig config)
    : runner_(std::move(runner)), config_(config), scheduler_(scheduler_config(config)) {
    // the engine's context may not exceed the model's or the runner's limit
    const bool within = runner_ && config.context >= 1 && config.context <= runner_->config().context &&
                        config.context <= runner_->context_limit();
    if (!within) throw std::invalid_argument("invalid engine configuration");
}

Engine::~Engine() {
    try {
        shutdown();
    } catch (...) {
    }
}

namespace {

// The submit checks, in the order the reference applies them (engine.cpp:19-26).
void validate_request(const Request& r, const std::set<RequestId>& seen, int context, int vocabulary) {
    const auto& g = r.generation;
    const std::uint64_t total = r.prompt_token_ids.size() + std::uint64_t(g.max_new_tokens);
    const bool shape_ok = !r.id.empty() && !seen.count(r.id) && !r.prompt_token_ids.empty() &&
                          g.max_new_tokens >= 1 && total <= std::uint64_t(context);
    if (!shape_ok) throw std::invalid_argument("invalid request, duplicate ID or context overflow");
    const auto outside = [vocabulary](TokenId t) { return t < 0 || t >= vocabulary; };
    if (std::any_of(r.prompt_token_ids.begin(), r.prompt_token_ids.end(), outside))
        throw std::invalid_argument("invalid prompt token");
    if (g.eos_token_id && outside(*g.eos_token_id)) throw std::invalid_argument("invalid EOS");
}

template <class Container>
void drop_finished(Container& states) {
    states.erase(std::remove_if(states.begin(), states.end(), [](const auto& s) { return s.finished; }),
                 states.end());
}

}  // namespace

void Engine::submit(Request request) {
    if (failed_) throw std::runtime_error("engine failed; create a new engine");
    validate_request(request, seen_, config_.context, runner_->config().vocabulary);
    seen_.insert(request.id);
    State state;
    state.request = std::move(request);
    waiting_.push_back(std::move(state));
}

void Engine::finish_host(State& state, TerminalCleanup cleanup) {
    if (state.resident && cleanup == TerminalCleanup::ReleaseSequence) runner_->release(state.request.id);
    runner_->release_reservation(state.request.id);
    state.resident = false;
    state.finished = true;
}

void Engine::terminal(State& state, FinishReason reason, std::optional<TokenId> token, const std::string& error,
                      TerminalCleanup cleanup) {
    if (state.finished) return;
    // Completion and cancellation give the pages back before the event; a fatal
    // failure leaves the cleanup to the runner (the reference's order,
    // engine.cpp:63-70).
    finish_host(state, cleanup);
    events_.push_back({state.request.id, token, reason, error});
}

void Engine::remove_finished(bool include_waiting) {
    drop_finished(active_);
    if (include_waiting) drop_finished(waiting_);
}

void Engine::restore_prefix(State& state) {
    const auto& id = state.request.id;
    const auto& prompt = state.request.prompt_token_ids;
    runner_->create(id);
    state.resident = true;
    const std::size_t cached = runner_->reuse_prefix(id, prompt);
    // A reused prefix must leave at least one prompt token to compute logits from,
    // and needs a paged runner (engine.cpp:44-55).
    const std::size_t page = runner_->kv_block_tokens();
    const bool usable = cached < prompt.size() && (cached == 0 || page != 0);
    if (!usable) throw std::runtime_error("invalid reusable prefix range");
    state.kv_block_tokens = page;
    state.prefilled = cached;
    step_stats_.prefix_reused_tokens += cached;
}

void Engine::resolve(std::vector<Outcome>& outcomes, std::size_t& resolved, const std::vector<SchedulePhase>& phases,
                     const std::vector<Saved>& saved, std::size_t events_before, const EngineStepStats& stats_before) {
    for (; resolved < outcomes.size(); ++resolved) {
        const Outcome& o = outcomes[resolved];
        State& s = active_[o.active_index];
        if (o.kind == Outcome::Error) {
            events_.push_back({s.request.id, std::nullopt, FinishReason::Error, o.message});
            continue;
        }
        const auto result = runner_->result(o.ticket);
        if (!result.finite) replay_and_fail(o.work_index, phases, outcomes, saved, events_before, stats_before);
        if (o.kind == Outcome::Chunk) continue;
        const TokenId token = result.token;
        const auto& r = s.request;
        if (r.generation.eos_token_id) {
            // Resolved right after its own append (see step()): decide as the reference does.
            s.output.back() = token;
            std::optional<FinishReason> finish;
            if (token == *r.generation.eos_token_id) finish = FinishReason::Eos;
            else if (s.output.size() == r.generation.max_new_tokens) finish = FinishReason::Length;
            if (finish) terminal(s, *finish, token);
            else events_.push_back({r.id, token, std::nullopt, {}});
            continue;
        }
        // Length finishes were applied to the runner at their turn; only the token was missing.
        s.output.back() = token;  // a request is scheduled at most once per step
        if (o.length_finish) events_.push_back({r.id, token, FinishReason::Length, {}});
        else events_.push_back({r.id, token, std::nullopt, {}});
    }
}

void Engine::replay_and_fail(std::size_t failing_work, const std::vector<SchedulePhase>& phases,
                             const std::vector<Outcome>& outcomes, const std::vector<Saved>& saved,
                             std::size_t events_before, const EngineStepStats& stats_before) {
    // Device results already known for the appends before the failing one.
    std::map<std::size_t, TokenId> known;
    for (const auto& o : outcomes)
        if (o.kind == Outcome::Token && o.work_index < failing_work) known[o.work_index] = runner_->result(o.ticket).token;
    step_failed_ = true;
    runner_->restore_batch();
    for (std::size_t i = 0; i < active_.size() && i < saved.size(); ++i) {
        auto& s = active_[i];
        s.prefilled = saved[i].prefilled;
        s.output.resize(saved[i].output_size);
        s.resident = saved[i].resident;
        s.finished = saved[i].finished;
    }
    events_.resize(events_before);
    step_stats_ = stats_before;
    runner_->set_replay(true);
    auto plan = scheduler_.plan(phases);
    const auto& order = plan.order();
    for (std::size_t w = 0; w < order.size(); ++w) {
        if (!plan.has_budget()) break;
        const auto& work = order[w];
        auto& s = active_[work.active_index];
        auto& r = s.request;
        try {
            if (!s.resident) restore_prefix(s);
            const bool prefilling = work.phase == SchedulePhase::Prefill;
            const auto count = plan.take_input(work.phase, r.prompt_token_ids.size() - s.prefilled);
            std::vector<TokenId> input;
            if (!prefilling) input = {s.output.back()};
            else
                input.assign(r.prompt_token_ids.begin() + std::ptrdiff_t(s.prefilled),
                             r.prompt_token_ids.begin() + std::ptrdiff_t(s.prefilled + count));
            if (w == failing_work) {
                runner_->set_replay(false);
                runner_->fail_append(r.id, input);  // throws the reference's failure
            }
            runner_->stage_append(r.id, input);
            if (prefilling) {
                s.prefilled += input.size();
                step_stats_.prefill_tokens += input.size();
            } else {
                step_stats_.decode_tokens += input.size();
            }
            if (s.prefilled < r.prompt_token_ids.size()) continue;
            runner_->cache_prefix(r.id);
            const TokenId token = known.at(w);
            s.output.push_back(token);
            std::optional<FinishReason> finish;
            if (r.generation.eos_token_id && token == *r.generation.eos_token_id) finish = FinishReason::Eos;
            else if (s.output.size() == r.generation.max_new_tokens) finish = FinishReason::Length;
            if (finish) terminal(s, *finish, token);
            else events_.push_back({r.id, token, std::nullopt, {}});
        } catch (const KvCapacityError& error) {
            terminal(s, FinishReason::Error, std::nullopt, error.what());
        }
    }
    runner_->set_replay(false);
    throw std::logic_error("batched step replay did not reach the failing append");
}

bool Engine::step() {
    step_stats_ = {};
    step_failed_ = false;
    if (failed_) throw std::runtime_error("engine failed");
    bool progressed = false;
    try {
        auto slots = scheduler_.admission_count(active_.size(), waiting_.size());
        while (slots && !waiting_.empty()) {
            auto& state = waiting_.front();
            const auto& request = state.request;
            // The final sampled token is delivered, never appended to KV.
            const auto tokens = request.prompt_token_ids.size() + std::size_t(request.generation.max_new_tokens) - 1;
            const auto admission = runner_->reserve_request(request.id, tokens);
            if (admission == KvAdmission::Wait && !active_.empty()) break;
            if (admission != KvAdmission::Ready) {
                terminal(state, FinishReason::Error, std::nullopt,
                         admission == KvAdmission::Impossible
                             ? "request exceeds total KV capacity"
                             : "KV capacity unavailable without active requests to make progress");
                waiting_.pop_front();
                progressed = true;
                continue;
            }
            active_.push_back(std::move(state));
            waiting_.pop_front();
            --slots;
            progressed = true;
        }
        if (active_.empty()) return progressed;
        std::vector<SchedulePhase> phases;
        phases.reserve(active_.size());
        for (const auto& state : active_)
            phases.push_back(state.output.empty() ? SchedulePhase::Prefill : SchedulePhase::Decode);
        std::vector<Saved> saved;
        saved.reserve(active_.size());
        for (const auto& s : active_) saved.push_back({s.prefilled, s.output.size(), s.resident, s.finished});
        const std::size_t events_before = events_.size();
        const EngineStepStats stats_before = step_stats_;
        runner_->begin_batch();
        auto plan = scheduler_.plan(phases);
        std::vector<Outcome> outcomes;
        outcomes.reserve(plan.order().size());
        std::size_t resolved = 0;
        const auto& order = plan.order();
        for (std::size_t w = 0; w < order.size(); ++w) {
            if (!plan.has_budget()) break;
            const auto& work = order[w];
            auto& s = active_[work.active_index];
            auto& r = s.request;
            try {
                if (!s.resident) restore_prefix(s);
                const bool prefilling = work.phase == SchedulePhase::Prefill;
                const auto count = plan.take_input(work.phase, r.prompt_token_ids.size() - s.prefilled);
                // one reused buffer: a decode append allocates nothing here
                std::vector<TokenId>& input = input_;
                if (!prefilling) input.assign(1, s.output.back());
                else
                    input.assign(r.prompt_token_ids.begin() + std::ptrdiff_t(s.prefilled),
                                 r.prompt_token_ids.begin() + std::ptrdiff_t(s.prefilled + count));
                const auto ticket = runner_->stage_append(r.id, input);
                if (prefilling) {
                    s.prefilled += input.size();
                    step_stats_.prefill_tokens += input.size();
                } else {
                    step_stats_.decode_tokens += input.size();
                }
                if (s.prefilled < r.prompt_token_ids.size()) {
                    outcomes.push_back({Outcome::Chunk, work.active_index, w, ticket, false, {}});
                    continue;
                }
                // Publish before sampling: the new output has no KV yet (engine.cpp:93-98).
                runner_->cache_prefix(r.id);
                s.output.push_back(0);  // the greedy token arrives with the device results
                Outcome o{Outcome::Token, work.active_index, w, ticket, false, {}};
                if (r.generation.eos_token_id) {
                    // Whether this request ends here depends on its token: resolve now.
                    outcomes.push_back(o);
                    runner_->flush();
                    resolve(outcomes, resolved, phases, saved, events_before, stats_before);
                    continue;
                }
                if (s.output.size() == r.generation.max_new_tokens) {
                    o.length_finish = true;
                    finish_host(s);
                }
                outcomes.push_back(o);
            } catch (const KvCapacityError& error) {
                // Request-scoped failure; a failed release still reaches the fatal handler.
                finish_host(s);
                outcomes.push_back({Outcome::Error, work.active_index, w, 0, false, error.what()});
            } catch (...) {
                // Appends before this request complete first, as they would have
                // (unless the failure is already the exact replayed one).
                if (!step_failed_) {
                    runner_->flush();
                    resolve(outcomes, resolved, phases, saved, events_before, stats_before);
                }
                throw;
            }
        }
        runner_->flush();
        resolve(outcomes, resolved, phases, saved, events_before, stats_before);
        runner_->end_batch();
        remove_finished();
    } catch (const std::exception& error) {
        // Poison first; backend ownership must survive a failed cleanup (engine.cpp:112-123).
        failed_ = true;
        std::string message = error.what();
        try {
            runner_->clear();
        } catch (const std::exception& cleanup) {
            message += "; cleanup failed: ";
            message += cleanup.what();
        } catch (...) {
            message += "; cleanup failed: unknown exception";
        }
        for (auto& s : active_) terminal(s, FinishReason::Error, std::nullopt, message, TerminalCleanup::RunnerManaged);
        for (auto& s : waiting_) terminal(s, FinishReason::Error, std::nullopt, message, TerminalCleanup::RunnerManaged);
        remove_finished(true);
    }
    return true;
}

std::vector<GenerationEvent> Engine::poll_events() {
    auto result = std::move(events_);
    events_.clear();
    return result;
}

void Engine::cancel(const RequestId& id) {
    for (auto& s : waiting_)
        if (s.request.id == id && !s.finished) {
            terminal(s, FinishReason::Cancelled);
            remove_finished(true);
            return;
        }
    for (auto& s : active_)
        if (s.request.id == id && !s.finished) {
            terminal(s, FinishReason::Cancelled);
            remove_finished();
            return;
        }
    throw std::invalid_argument("request is unknown or already terminal");
}

void Engine::shutdown() {
    try {
        for (auto& s : active_) terminal(s, FinishReason::Cancelled);
        for (auto& s : waiting_) terminal(s, FinishReason::Cancelled);
    } catch (...) {
        remove_finished(true);
        throw;
    }
    remove_finished(true);
    runner_->clear();
}

}  // namespace miniprefix_b200
