#include "protocol.h"

#include <iomanip>
#include <sstream>
#include <stdexcept>

namespace miniprefix_b200::protocol {
namespace {

int read_int(std::istringstream& in) {
    int n;
    if (!(in >> n)) throw std::invalid_argument("missing integer");
    return n;
}

std::vector<TokenId> read_tokens(std::istringstream& in, int count) {
    if (count < 1 || count > 131072) throw std::invalid_argument("invalid token count");
    std::vector<TokenId> tokens;
    tokens.reserve(std::size_t(count));
    for (int i = 0; i < count; ++i) tokens.push_back(read_int(in));
    return tokens;
}

bool diagnostic(Kind k) {
    return k == Kind::Forward || k == Kind::Reuse || k == Kind::Cache || k == Kind::Release ||
           k == Kind::ClearPrefix || k == Kind::CostTiming;
}

}  // namespace

Command parse(const std::string& line) {
    std::istringstream in(line);
    std::string op;
    in >> op;
    Command c;
    if (op == "SUBMIT") {
        const int id = read_int(in), limit = read_int(in), eos = read_int(in), n = read_int(in);
        if (id < 1 || limit < 1) throw std::invalid_argument("invalid request");
        c.kind = Kind::Submit;
        c.request.id = std::to_string(id);
        c.request.prompt_token_ids = read_tokens(in, n);
        c.request.generation.max_new_tokens = std::uint32_t(limit);
        if (eos >= 0) c.request.generation.eos_token_id = eos;
        else if (eos != -1) throw std::invalid_argument("invalid EOS");
        return c;
    }
    if (op == "FORWARD" || op == "REUSE") {
        c.kind = op == "FORWARD" ? Kind::Forward : Kind::Reuse;
        c.id = read_int(in);
        const int n = read_int(in);
        c.input = read_tokens(in, n);
        if (c.id < 1) throw std::invalid_argument("invalid diagnostic sequence");
        return c;
    }
    if (op == "CANCEL" || op == "CACHE" || op == "RELEASE") {
        c.kind = op == "CANCEL" ? Kind::Cancel : (op == "CACHE" ? Kind::Cache : Kind::Release);
        c.id = read_int(in);
        return c;
    }
    if (op == "COST_TIMING") {
        c.kind = Kind::CostTiming;
        c.id = read_int(in);
        if (c.id != 0 && c.id != 1) throw std::invalid_argument("invalid timing flag");
        return c;
    }
    if (op == "STEP") c.kind = Kind::Step;
    else if (op == "STEP_STATS") c.kind = Kind::StepStats;
    else if (op == "CLEAR_PREFIX") c.kind = Kind::ClearPrefix;
    else if (op == "COST_STATS") c.kind = Kind::CostStats;
    else if (op == "STATS") c.kind = Kind::Stats;
    else if (op == "QUIT") c.kind = Kind::Quit;
    else throw std::invalid_argument("unknown command");
    return c;
}

void ready(std::ostream& out, int vocabulary, int eos, int context, const std::string& backend) {
    out << "READY MINIPREFIX 3 " << vocabulary << ' ' << eos << ' ' << context << ' ' << backend << '\n' << std::flush;
}
void ok(std::ostream& out) { out << "OK\n"; }
void count(std::ostream& out, std::size_t value) { out << "OK " << value << '\n'; }
void logits(std::ostream& out, const std::vector<float>& values) {
    out << "OK" << std::setprecision(9);
    for (float v : values) out << ' ' << v;
    out << '\n';
}
void events(std::ostream& out, const std::vector<GenerationEvent>& batch) {
    out << "OK " << batch.size();
    for (const auto& e : batch)
        out << ' ' << e.request_id << ' ' << (e.token_id ? *e.token_id : -1) << ' '
            << (e.finish_reason ? static_cast<int>(*e.finish_reason) : -1);
    out << '\n';
}
void stats(std::ostream& out, const RunnerStats& s) {
    const std::size_t v[] = {s.live_sequences, s.live_kv_bytes, s.peak_kv_bytes, s.forward_tokens,
                             s.device_weight_bytes, s.weight_uploaded_bytes, s.token_uploaded_bytes,
                             s.kv_uploaded_bytes, s.logits_downloaded_bytes, s.device_allocations,
                             s.device_workspace_bytes, s.kv_block_tokens, s.kv_total_blocks, s.kv_live_blocks,
                             s.kv_peak_blocks, s.kv_reserved_bytes, s.block_table_uploaded_bytes,
                             s.block_table_device_bytes, s.prefix_cache_capacity, s.kv_cached_blocks,
                             s.kv_cache_only_blocks, s.prefix_hits, s.prefix_misses, s.prefix_reused_tokens,
                             s.prefix_evictions};
    out << "OK";
    for (std::size_t x : v) out << ' ' << x;
    out << '\n';
}
void cost_stats(std::ostream& out, const CostStats& s) {
    out << "OK " << s.lookup_calls << ' ' << s.lookup_ns << ' ' << s.publish_calls << ' ' << s.publish_ns << ' '
        << s.cow_pages << ' ' << s.cow_bytes << ' ' << s.cow_copy_ns << ' ' << s.cow_timed_copies << '\n';
}
void step_stats(std::ostream& out, const EngineStepStats& s) {
    out << "OK " << s.prefix_reused_tokens << ' ' << s.prefill_tokens << ' ' << s.decode_tokens << '\n';
}
void error(std::ostream& out, const std::string& message) { out << "ERROR " << message << '\n'; }

std::string Diagnostics::key(int id) { return "reference/" + std::to_string(id); }

std::string Diagnostics::ensure(int id) {
    std::string name = key(id);
    if (!created_.count(name)) {
        runner_.create(name);
        created_.insert(name);
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

int serve(Engine& engine, std::istream& in, std::ostream& out) {
    Diagnostics diag(engine.runner());
    std::string line;
    while (std::getline(in, line)) {
        try {
            Command command = parse(line);
            // the runner is shared with the engine: once the engine has failed, no
            // direct runner command may use it again
            if (engine.failed() && diagnostic(command.kind))
                throw std::runtime_error("engine failed; create a new engine");
            switch (command.kind) {
                case Kind::Submit:
                    engine.submit(std::move(command.request));
                    ok(out);
                    break;
                case Kind::Step:
                    engine.step();
                    events(out, engine.poll_events());
                    break;
                case Kind::StepStats: step_stats(out, engine.last_step_stats()); break;
                case Kind::Cancel:
                    engine.cancel(std::to_string(command.id));
                    events(out, engine.poll_events());
                    break;
                case Kind::ClearPrefix:
                    diag.clear_prefix();
                    ok(out);
                    break;
                case Kind::Cache:
                    diag.cache(command.id);
                    ok(out);
                    break;
                case Kind::Reuse: count(out, diag.reuse(command.id, command.input)); break;
                case Kind::Forward: logits(out, diag.forward(command.id, command.input)); break;
                case Kind::Release:
                    diag.release(command.id);
                    ok(out);
                    break;
                case Kind::CostStats: cost_stats(out, engine.runner().cost_stats()); break;
                case Kind::CostTiming:
                    engine.runner().set_cost_timing(command.id != 0);
                    ok(out);
                    break;
                case Kind::Stats: stats(out, engine.runner().stats()); break;
                case Kind::Quit:
                    engine.shutdown();
                    ok(out);
                    out << std::flush;
                    return 0;
            }
        } catch (const std::exception& e) {
            error(out, e.what());
        }
        out << std::flush;
    }
    return 0;
}

}  // namespace miniprefix_b200::protocol
