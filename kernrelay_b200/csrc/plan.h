// Schedule executor behind kr_plan_run (reference: exec/exec_main.cpp RunPlanCli).
#pragma once

#include <string>

namespace krb {
namespace plan {

// Runs the schedule at `schedule_path` (the reference scheduler's schedule.json) on the
// devices in `devices` ("" = 0..nranks-1) in `mode` (direct / graph / graph_per_stream /
// graph_segment), `warmup` untimed and `iters` timed runs, and writes the result JSON to
// `out_path`.  Returns the result JSON; throws std::runtime_error on any failure.
std::string run(const std::string &schedule_path, int iters, int warmup,
                const std::string &devices, const std::string &mode, const std::string &out_path);

// Parses and validates the schedule without touching a GPU; returns a JSON summary
// (nodes, tasks, lanes, publishes) or throws with the executor's error message.
std::string check(const std::string &schedule_path);

}  // namespace plan
}  // namespace krb
