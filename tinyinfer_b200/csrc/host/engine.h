// Request lifecycle and the per-step loop: the reference Engine
// (miniprefix/include/miniprefix/engine.h, miniprefix/src/engine/engine.cpp) with
// identical admission, scheduling, prefix restore, publish-before-sample, greedy
// sampling (first maximum), finish reasons, events and failure handling -- but
// all appends of one step run as one device forward through the runner's
// staged batch interface (model_runner.h).
//
// Every host decision of a step is taken in the reference's order, request by
// request; only the device results (greedy token, finiteness) arrive later.
// Events are queued in that same order. A request with an EOS token forces its
// result before the next request is processed (its finish could change later
// decisions). When a forward reports a nonfinite result, the whole step's host
// state is restored from the runner checkpoint and replayed up to the failing
// request, whose append then fails exactly as the reference's does
// (engine.cpp:112-123): the engine is poisoned and every request ends in Error.
#pragma once
#include <deque>
#include <memory>
#include <set>

#include "model_runner.h"
#include "scheduler.h"

namespace miniprefix_b200 {

class Engine {
public:
    Engine(std::unique_ptr<ModelRunner> runner, EngineConfig config);
    ~Engine();
    void submit(Request request);
    bool step();
    std::vector<GenerationEvent> poll_events();
    void cancel(const RequestId& id);
    void shutdown();
    bool idle() const { return active_.empty() && waiting_.empty(); }
    bool failed() const { return failed_; }
    ModelRunner& runner() { return *runner_; }
    const EngineStepStats& last_step_stats() const { return step_stats_; }

private:
    struct State {
        Request request;
        std::size_t prefilled = 0, kv_block_tokens = 0;
        std::vector<TokenId> output;
        bool resident = false, finished = false;
    };
    enum class TerminalCleanup { ReleaseSequence, RunnerManaged };
    // One queued outcome of the current step, resolved in plan order.
    struct Outcome {
        enum Kind { Chunk, Token, Error } kind;
        std::size_t active_index;
        std::size_t work_index;  // position in the step's plan order
        std::size_t ticket = 0;
        bool length_finish = false;
        std::string message;
    };
    struct Saved {
        std::size_t prefilled;
        std::size_t output_size;
        bool resident, finished;
    };

    void restore_prefix(State& state);
    void terminal(State& state, FinishReason reason, std::optional<TokenId> token = std::nullopt,
                  const std::string& error = "", TerminalCleanup cleanup = TerminalCleanup::ReleaseSequence);
    // The runner/reservation half of terminal(); the event is queued separately.
    void finish_host(State& state, TerminalCleanup cleanup = TerminalCleanup::ReleaseSequence);
    void remove_finished(bool include_waiting = false);
    void resolve(std::vector<Outcome>& outcomes, std::size_t& resolved, const std::vector<SchedulePhase>& phases,
                 const std::vector<Saved>& saved, std::size_t events_before, const EngineStepStats& stats_before);
    [[noreturn]] void replay_and_fail(std::size_t failing_work, const std::vector<SchedulePhase>& phases,
                                      const std::vector<Outcome>& outcomes, const std::vector<Saved>& saved,
                                      std::size_t events_before, const EngineStepStats& stats_before);

    std::unique_ptr<ModelRunner> runner_;
    EngineConfig config_;
    Scheduler scheduler_;
    std::deque<State> waiting_;
    std::vector<State> active_;
    std::set<RequestId> seen_;
    std::vector<GenerationEvent> events_;
    std::vector<TokenId> input_;  // the input tokens of the append being staged
    bool failed_ = false;
    bool step_failed_ = false;  // a failed append of this step was replayed and rethrown
    EngineStepStats step_stats_;
};

}  // namespace miniprefix_b200
