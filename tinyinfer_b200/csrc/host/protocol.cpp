#include "protocol.h"

#include <iomanip>
#include <sstream>
#include <stdexcept>

namespace miniprefix_b200::protocol {
namespace {

// The fields of one request line, left to right. Numbers use formatted
// extraction, so "+1" and "1x" both read 1 and anything after a number is left
// for the next read.
class Fields {
public:
    explicit Fields(const std::string& line) : in_(line) {}
    std::string verb() {
        std::string w;
        in_ >> w;
        return w;
    }
    int number() {
        int n;
        if (!(in_ >> n)) throw std::invalid_argument("missing integer");
        return n;
    }
    std::vector<TokenId> token_list(int count) {
        if (count < 1 || count > kMaxTokens) throw std::invalid_argument("invalid token count");
        std::vector<TokenId> out(static_cast<std::size_t>(count));
        for (auto& t : out) t = number();
        return out;
    }

private:
    static constexpr int kMaxTokens = 131072;
    std::istringstream in_;
};

// Per-verb grammars. Each reads its fields in wire order and applies its checks
// at the point the wire format defines them (e.g. SUBMIT validates id and limit
// before reading the tokens, and the EOS field only after them).
void fields_submit(Fields& f, Command& c) {
    const int id = f.number(), limit = f.number(), eos = f.number(), n = f.number();
    if (id < 1 || limit < 1) throw std::invalid_argument("invalid request");
    c.request.id = std::to_string(id);
    c.request.prompt_token_ids = f.token_list(n);
    c.request.generation.max_new_tokens = static_cast<std::uint32_t>(limit);
    if (eos < -1) throw std::invalid_argument("invalid EOS");
    if (eos >= 0) c.request.generation.eos_token_id = eos;
}
void fields_sequence_input(Fields& f, Command& c) {  // FORWARD / REUSE id count tokens
    c.id = f.number();
    const int n = f.number();
    c.input = f.token_list(n);
    if (c.id < 1) throw std::invalid_argument("invalid diagnostic sequence");
}
void fields_id(Fields& f, Command& c) { c.id = f.number(); }
void fields_flag(Fields& f, Command& c) {
    c.id = f.number();
    if (c.id != 0 && c.id != 1) throw std::invalid_argument("invalid timing flag");
}
void fields_none(Fields&, Command&) {}

struct Verb {
    const char* word;
    Kind kind;
    void (*read)(Fields&, Command&);
};
constexpr Verb kVerbs[] = {
    {"SUBMIT", Kind::Submit, fields_submit},
    {"FORWARD", Kind::Forward, fields_sequence_input},
    {"REUSE", Kind::Reuse, fields_sequence_input},
    {"CANCEL", Kind::Cancel, fields_id},
    {"CACHE", Kind::Cache, fields_id},
    {"RELEASE", Kind::Release, fields_id},
    {"STEP", Kind::Step, fields_none},
    {"STEP_STATS", Kind::StepStats, fields_none},
    {"CLEAR_PREFIX", Kind::ClearPrefix, fields_none},
    {"COST_STATS", Kind::CostStats, fields_none},
    {"COST_TIMING", Kind::CostTiming, fields_flag},
    {"STATS", Kind::Stats, fields_none},
    {"QUIT", Kind::Quit, fields_none},
};

// Commands that call the runner directly rather than through the engine.
bool direct_runner_call(Kind k) {
    switch (k) {
        case Kind::Forward:
        case Kind::Reuse:
        case Kind::Cache:
        case Kind::Release:
        case Kind::ClearPrefix:
        case Kind::CostTiming: return true;
        default: return false;
    }
}

// "OK" followed by each value, space-separated, one line.
template <class It>
void ok_line(std::ostream& out, It first, It last) {
    out << "OK";
    for (; first != last; ++first) out << ' ' << *first;
    out << '\n';
}

// Wire order of the 25 RunnerStats fields and the 8 CostStats fields.
constexpr std::size_t RunnerStats::*kRunnerWire[] = {
    &RunnerStats::live_sequences,        &RunnerStats::live_kv_bytes,
    &RunnerStats::peak_kv_bytes,         &RunnerStats::forward_tokens,
    &RunnerStats::device_weight_bytes,   &RunnerStats::weight_uploaded_bytes,
    &RunnerStats::token_uploaded_bytes,  &RunnerStats::kv_uploaded_bytes,
    &RunnerStats::logits_downloaded_bytes, &RunnerStats::device_allocations,
    &RunnerStats::device_workspace_bytes, &RunnerStats::kv_block_tokens,
    &RunnerStats::kv_total_blocks,       &RunnerStats::kv_live_blocks,
    &RunnerStats::kv_peak_blocks,        &RunnerStats::kv_reserved_bytes,
    &RunnerStats::block_table_uploaded_bytes, &RunnerStats::block_table_device_bytes,
    &RunnerStats::prefix_cache_capacity, &RunnerStats::kv_cached_blocks,
    &RunnerStats::kv_cache_only_blocks,  &RunnerStats::prefix_hits,
    &RunnerStats::prefix_misses,         &RunnerStats::prefix_reused_tokens,
    &RunnerStats::prefix_evictions,
};
constexpr std::uint64_t CostStats::*kCostWire[] = {
    &CostStats::lookup_calls, &CostStats::lookup_ns, &CostStats::publish_calls,  &CostStats::publish_ns,
    &CostStats::cow_pages,    &CostStats::cow_bytes, &CostStats::cow_copy_ns,    &CostStats::cow_timed_copies,
};

}  // namespace

Command parse(const std::string& line) {
    Fields f(line);
    const std::string word = f.verb();
    for (const Verb& v : kVerbs) {
        if (word != v.word) continue;
        Command c;
        c.kind = v.kind;
        v.read(f, c);
        return c;
    }
    throw std::invalid_argument("unknown command");
}

void ready(std::ostream& out, int vocabulary, int eos, int context, const std::string& backend) {
    out << "READY MINIPREFIX 3 " << vocabulary << ' ' << eos << ' ' << context << ' ' << backend << '\n' << std::flush;
}
void ok(std::ostream& out) { out << "OK\n"; }
void count(std::ostream& out, std::size_t value) {
    const std::size_t v[] = {value};
    ok_line(out, std::begin(v), std::end(v));
}
void logits(std::ostream& out, const std::vector<float>& values) {
    out << std::setprecision(9);  // enough digits to round-trip a float
    ok_line(out, values.begin(), values.end());
}
void events(std::ostream& out, const std::vector<GenerationEvent>& batch) {
    out << "OK " << batch.size();
    for (const auto& e : batch) {
        const int token = e.token_id ? *e.token_id : -1;
        const int reason = e.finish_reason ? static_cast<int>(*e.finish_reason) : -1;
        out << ' ' << e.request_id << ' ' << token << ' ' << reason;
    }
    out << '\n';
}
void stats(std::ostream& out, const RunnerStats& s) {
    std::vector<std::size_t> v;
    v.reserve(std::size(kRunnerWire));
    for (auto field : kRunnerWire) v.push_back(s.*field);
    ok_line(out, v.begin(), v.end());
}
void cost_stats(std::ostream& out, const CostStats& s) {
    std::vector<std::uint64_t> v;
    v.reserve(std::size(kCostWire));
    for (auto field : kCostWire) v.push_back(s.*field);
    ok_line(out, v.begin(), v.end());
}
void step_stats(std::ostream& out, const EngineStepStats& s) {
    const std::size_t v[] = {s.prefix_reused_tokens, s.prefill_tokens, s.decode_tokens};
    ok_line(out, std::begin(v), std::end(v));
}
void error(std::ostream& out, const std::string& message) { out << "ERROR " << message << '\n'; }

std::string Diagnostics::key(int id) { return "reference/" + std::to_string(id); }

std::string Diagnostics::ensure(int id) {
    std::string name = key(id);
    if (created_.insert(name).second) {
        try {
            runner_.create(name);
        } catch (...) {
            created_.erase(name);
            throw;
        }
    }
    return name;
}

std::vector<float> Diagnostics::forward(int id, const std::vector<TokenId>& tokens) {
    return runner_.append(ensure(id), tokens);
}
std::size_t Diagnostics::reuse(int id, const std::vector<TokenId>& tokens) {
    return runner_.reuse_prefix(ensure(id), tokens);
}
void Diagnostics::cache(int id) { runner_.cache_prefix(key(id)); }
void Diagnostics::release(int id) {
    const std::string name = key(id);
    runner_.release(name);
    created_.erase(name);
}
void Diagnostics::clear_prefix() { runner_.clear_prefix_cache(); }

namespace {

// One connection: executes parsed commands against the engine (or, for the
// diagnostics, its runner) and writes one response line per command.
class Session {
public:
    Session(Engine& engine, std::ostream& out) : engine_(engine), diag_(engine.runner()), out_(out) {}

    // false once QUIT has been served
    bool execute(Command& c) {
        // the runner is shared with the engine: after the engine failed, no
        // direct runner call may use it again
        if (engine_.failed() && direct_runner_call(c.kind)) throw std::runtime_error("engine failed; create a new engine");
        (this->*kHandlers[static_cast<int>(c.kind)])(c);
        return c.kind != Kind::Quit;
    }

private:
    void submit(Command& c) {
        engine_.submit(std::move(c.request));
        ok(out_);
    }
    void step(Command&) {
        engine_.step();
        events(out_, engine_.poll_events());
    }
    void step_stats_(Command&) { step_stats(out_, engine_.last_step_stats()); }
    void cancel(Command& c) {
        engine_.cancel(std::to_string(c.id));
        events(out_, engine_.poll_events());
    }
    void clear_prefix(Command&) {
        diag_.clear_prefix();
        ok(out_);
    }
    void cache(Command& c) {
        diag_.cache(c.id);
        ok(out_);
    }
    void reuse(Command& c) { count(out_, diag_.reuse(c.id, c.input)); }
    void forward(Command& c) { logits(out_, diag_.forward(c.id, c.input)); }
    void release(Command& c) {
        diag_.release(c.id);
        ok(out_);
    }
    void stats_(Command&) { stats(out_, engine_.runner().stats()); }
    void cost_stats_(Command&) { cost_stats(out_, engine_.runner().cost_stats()); }
    void cost_timing(Command& c) {
        engine_.runner().set_cost_timing(c.id != 0);
        ok(out_);
    }
    void quit(Command&) {
        engine_.shutdown();
        ok(out_);
    }

    using Handler = void (Session::*)(Command&);
    // indexed by Kind, in its declaration order
    static constexpr Handler kHandlers[] = {
        &Session::submit,      &Session::step,    &Session::step_stats_, &Session::cancel,
        &Session::clear_prefix, &Session::cache,  &Session::reuse,       &Session::forward,
        &Session::release,     &Session::stats_,  &Session::cost_stats_, &Session::cost_timing,
        &Session::quit,
    };
    static_assert(std::size(kHandlers) == static_cast<std::size_t>(Kind::Quit) + 1, "one handler per Kind");

    Engine& engine_;
    Diagnostics diag_;
    std::ostream& out_;
};

}  // namespace

int serve(Engine& engine, std::istream& in, std::ostream& out) {
    Session session(engine, out);
    for (std::string line; std::getline(in, line);) {
        bool more = true;
        try {
            Command c = parse(line);
            more = session.execute(c);
        } catch (const std::exception& e) {
            error(out, e.what());
        }
        out << std::flush;
        if (!more) break;
    }
    return 0;
}

}  // namespace miniprefix_b200::protocol
