// Worker protocol v3: the line protocol of the reference worker
// (miniprefix/apps/protocol/*, miniprefix/apps/worker.cpp), on this engine.
//
// Requests, one per line (fields separated by whitespace; trailing fields are
// ignored; integers are read with formatted extraction, so "+1" and "1x" read 1):
//   SUBMIT id max_new eos count t1..tcount   eos -1: none
//   STEP | STEP_STATS | STATS | COST_STATS | CLEAR_PREFIX | QUIT
//   CANCEL id | CACHE id | RELEASE id | COST_TIMING 0|1
//   FORWARD id count t1..tcount | REUSE id count t1..tcount
// FORWARD / REUSE / CACHE / RELEASE act directly on the runner, on sequences
// named "reference/<id>" (a namespace apart from the engine's request ids).
// Responses: "OK", "OK n", "OK logits..." (9 significant digits), events
// "OK n (id token reason)*" (-1 for none), the 25 RunnerStats / 8 CostStats / 3
// step-stats fields, or "ERROR message"; the stream is flushed after each line.
// Once the engine has failed, the runner diagnostics answer
// "ERROR engine failed; create a new engine".
#pragma once
#include <istream>
#include <ostream>
#include <set>
#include <string>
#include <vector>

#include "engine.h"

namespace miniprefix_b200::protocol {

enum class Kind { Submit, Step, StepStats, Cancel, ClearPrefix, Cache, Reuse, Forward, Release, Stats, CostStats,
                  CostTiming, Quit };

struct Command {
    Kind kind = Kind::Step;
    int id = 0;
    Request request;
    std::vector<TokenId> input;
};

// Throws std::invalid_argument with the protocol's messages, validating in the
// order the wire format defines.
Command parse(const std::string& line);

void ready(std::ostream& out, int vocabulary, int eos, int context, const std::string& backend);
void ok(std::ostream& out);
void count(std::ostream& out, std::size_t value);
void logits(std::ostream& out, const std::vector<float>& values);
void events(std::ostream& out, const std::vector<GenerationEvent>& batch);
void stats(std::ostream& out, const RunnerStats& s);
void cost_stats(std::ostream& out, const CostStats& s);
void step_stats(std::ostream& out, const EngineStepStats& s);
void error(std::ostream& out, const std::string& message);

// The direct runner commands. A sequence is created on its first FORWARD or
// REUSE and kept when that append or reuse fails.
class Diagnostics {
public:
    explicit Diagnostics(ModelRunner& runner) : runner_(runner) {}
    std::vector<float> forward(int id, const std::vector<TokenId>& tokens);
    std::size_t reuse(int id, const std::vector<TokenId>& tokens);
    void cache(int id);
    void release(int id);
    void clear_prefix();

private:
    static std::string key(int id);
    std::string ensure(int id);
    ModelRunner& runner_;
    std::set<std::string> created_;
};

// Serves lines until QUIT (which shuts the engine down) or end of input.
int serve(Engine& engine, std::istream& in, std::ostream& out);

}  // namespace miniprefix_b200::protocol
