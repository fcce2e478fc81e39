// Admission and per-step order/budget: the reference Scheduler/SchedulePlan
// (miniprefix/include/miniprefix/scheduler.h:13-32, miniprefix/src/scheduler/
// scheduler.cpp:10-32): decodes first then prefills, each in active order; a
// decode takes one token, a prefill min(unprefilled, chunk, remaining budget).
#pragma once
#include <cstddef>
#include <vector>

namespace miniprefix_b200 {

enum class SchedulePhase { Prefill, Decode };
struct ScheduledRequest {
    std::size_t active_index;
    SchedulePhase phase;
};
struct SchedulerConfig {
    int max_batch_size = 2, token_budget = 32, prefill_chunk = 16;
};

class SchedulePlan {
    friend class Scheduler;
    std::vector<ScheduledRequest> order_;
    std::size_t remaining_, chunk_;
    SchedulePlan(const std::vector<SchedulePhase>& phases, const SchedulerConfig& config);

public:
    const std::vector<ScheduledRequest>& order() const { return order_; }
    bool has_budget() const { return remaining_ != 0; }
    std::size_t take_input(SchedulePhase phase, std::size_t unprefilled_tokens);
};

class Scheduler {
    SchedulerConfig config_;

public:
    explicit Scheduler(SchedulerConfig config);
    std::size_t admission_count(std::size_t active, std::size_t waiting) const;
    SchedulePlan plan(const std::vector<SchedulePhase>& active_phases) const { return SchedulePlan(active_phases, config_); }
};

}  // namespace miniprefix_b200
