// Fixture generator: runs the reference's own scheduler simulation (run_paged over the reference's
// KVManager, compiled from its sources) on seeded workloads and prints, per scenario, the workload, the
// configuration, the reference's metrics and the decision stream recorded by TracingKVManager.  Built and run
// by make_sim_traces.py; not part of the library.
#include <cstdio>
#include <string>
#include <vector>

#include "kvpage/simulator.h"
#include "kvpage/workload.h"
#include "tracing_kv_manager.h"

using namespace kvp;

namespace {

struct Scenario {
    const char* name;
    WorkloadConfig w;
    SimConfig c;
};

std::vector<Scenario> scenarios() {
    std::vector<Scenario> out;
    {  // FCFS, swap preemption, persistent prefix cache, two samples per request (fork + copy-on-write)
        Scenario s{"fcfs_swap_cache_forks", {}, {}};
        s.w.seed = 11;
        s.w.num_requests = 36;
        s.w.mean_interarrival = 0.5;
        s.w.prompt_min = 20;
        s.w.prompt_max = 120;
        s.w.output_min = 10;
        s.w.output_max = 80;
        s.w.shared_prefix_fraction = 0.5;
        s.w.prefix_len = 48;
        s.w.num_prefix_groups = 2;
        s.w.samples_per_request = 2;
        s.w.max_seq_len = 256;
        s.c.num_blocks = 96;
        s.c.block_size = 16;
        s.c.preempt_mode = PreemptMode::Swap;
        s.c.prefix_cache = true;
        s.c.swap_blocks_per_step = 8;
        s.c.prefill_tokens_per_step = 256;
        out.push_back(s);
    }
    {  // shortest-prompt-first, recompute preemption, long-tail prompts with shared prefixes
        Scenario s{"spf_recompute_prefix", {}, {}};
        s.w.seed = 12;
        s.w.num_requests = 48;
        s.w.mean_interarrival = 0.3;
        s.w.prompt_dist = Dist::LongTail;
        s.w.prompt_min = 16;
        s.w.prompt_max = 160;
        s.w.output_min = 8;
        s.w.output_max = 64;
        s.w.shared_prefix_fraction = 0.5;
        s.w.prefix_len = 40;
        s.w.num_prefix_groups = 3;
        s.w.max_seq_len = 256;
        s.c.num_blocks = 64;
        s.c.block_size = 16;
        s.c.policy = Policy::ShortestPromptFirst;
        s.c.preempt_mode = PreemptMode::Recompute;
        out.push_back(s);
    }
    {  // priority classes with displacement; swap pool too small for every victim (recompute fallback);
       // block size 8
        Scenario s{"priority_swap_capacity_b8", {}, {}};
        s.w.seed = 13;
        s.w.num_requests = 40;
        s.w.mean_interarrival = 0.4;
        s.w.prompt_min = 10;
        s.w.prompt_max = 90;
        s.w.output_min = 10;
        s.w.output_max = 70;
        s.w.high_priority_fraction = 0.3;
        s.w.shared_prefix_fraction = 0.4;
        s.w.prefix_len = 24;
        s.w.samples_per_request = 2;
        s.w.max_seq_len = 200;
        s.c.num_blocks = 120;
        s.c.block_size = 8;
        s.c.policy = Policy::Priority;
        s.c.preempt_mode = PreemptMode::Swap;
        s.c.swap_capacity_blocks = 24;
        s.c.prefix_cache = true;
        out.push_back(s);
    }
    {  // serving scale (the data-plane benchmark's stream): long-tail prompts, shared prefixes, FCFS, swap
        Scenario s{"serving_fcfs_swap", {}, {}};
        s.w.seed = 21;
        s.w.num_requests = 256;
        s.w.mean_interarrival = 0.25;
        s.w.prompt_dist = Dist::LongTail;
        s.w.prompt_min = 256;
        s.w.prompt_max = 3072;
        s.w.output_min = 32;
        s.w.output_max = 160;
        s.w.shared_prefix_fraction = 0.3;
        s.w.prefix_len = 512;
        s.w.num_prefix_groups = 4;
        s.w.max_seq_len = 3300;
        s.c.num_blocks = 3072;
        s.c.block_size = 16;
        s.c.preempt_mode = PreemptMode::Swap;
        s.c.prefix_cache = true;
        out.push_back(s);
    }
    return out;
}

}  // namespace

int main() {
    for (const Scenario& s : scenarios()) {
        trace_rows().clear();
        const std::vector<Request> reqs = generate_workload(s.w);
        const Metrics m = run_paged(reqs, s.c);
        std::printf("scenario %s\n", s.name);
        std::printf("config %d %d %d %d %d %d %d %d %d %d %d\n", s.c.num_blocks, s.c.block_size,
                    static_cast<int>(s.c.policy), s.c.watermark_blocks, s.c.max_running,
                    static_cast<int>(s.c.preempt_mode), s.c.swap_capacity_blocks, s.c.prefill_tokens_per_step,
                    s.c.swap_blocks_per_step, s.c.prefix_cache ? 1 : 0, s.c.fork_sharing ? 1 : 0);
        for (const Request& r : reqs)
            std::printf("request %lld %d %d %d %d %d %lld %d\n", static_cast<long long>(r.id), r.arrival,
                        r.prompt_len, r.output_len, r.prefix_group, r.prefix_len, static_cast<long long>(r.fork_of),
                        r.priority);
        std::printf("metrics %lld %lld %lld %lld %lld %lld %lld %lld %lld %lld %d\n",
                    static_cast<long long>(m.total_steps), static_cast<long long>(m.tokens_generated),
                    static_cast<long long>(m.preemptions), static_cast<long long>(m.recomputed_tokens),
                    static_cast<long long>(m.cow_copies), static_cast<long long>(m.swap_out_blocks),
                    static_cast<long long>(m.swap_in_blocks), static_cast<long long>(m.cache_hits),
                    static_cast<long long>(m.cache_evictions), static_cast<long long>(m.prefill_tokens_computed),
                    m.requests_completed);
        for (const auto& row : trace_rows())
            std::printf("row %lld %lld %lld %lld %lld %lld\n", static_cast<long long>(row[0]),
                        static_cast<long long>(row[1]), static_cast<long long>(row[2]),
                        static_cast<long long>(row[3]), static_cast<long long>(row[4]),
                        static_cast<long long>(row[5]));
        std::printf("end\n");
    }
    return 0;
}
