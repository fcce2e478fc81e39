#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace miniprefix_b200 {

Scheduler::Scheduler(SchedulerConfig config) : config_(config) {
    if (config.max_batch_size < 1 || config.token_budget < 1 || config.prefill_chunk < 1)
        throw std::invalid_argument("invalid scheduler configuration");
}

std::size_t Scheduler::admission_count(std::size_t active, std::size_t waiting) const {
    const std::size_t capacity = std::size_t(config_.max_batch_size);
    return active >= capacity ? 0 : std::min(waiting, capacity - active);
}

SchedulePlan::SchedulePlan(const std::vector<SchedulePhase>& phases, const SchedulerConfig& config)
    : remaining_(std::size_t(config.token_budget)), chunk_(std::size_t(config.prefill_chunk)) {
    order_.reserve(phases.size());
    for (std::size_t i = 0; i < phases.size(); ++i)
        if (phases[i] == SchedulePhase::Decode) order_.push_back({i, SchedulePhase::Decode});
    for (std::size_t i = 0; i < phases.size(); ++i)
        if (phases[i] == SchedulePhase::Prefill) order_.push_back({i, SchedulePhase::Prefill});
}

std::size_t SchedulePlan::take_input(SchedulePhase phase, std::size_t unprefilled_tokens) {
    if (!remaining_) return 0;
    if (phase == SchedulePhase::Prefill && !unprefilled_tokens)
        throw std::invalid_argument("prefill requires an uncached suffix");
    const std::size_t count =
        phase == SchedulePhase::Decode ? 1 : std::min({unprefilled_tokens, chunk_, remaining_});
    remaining_ -= count;
    return count;
}

}  // namespace miniprefix_b200
