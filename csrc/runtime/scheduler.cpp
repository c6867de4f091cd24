// Coordinator scheduling decisions (reference coordinator/src/state.rs:63-225, routes.rs:244-263):
//
//   push acceptance  reject when staleness = max(acc_version - push_version, 0) exceeds the maximum, or when
//                    the node already has a contribution with seq_num >= the pushed one (dedup); otherwise
//                    accept with weight tokens * decay^staleness (the caller replaces the node's older
//                    contribution)
//   merge trigger    at least one contribution; at least max(active/2, 2) of them (1 with a single active
//                    node; an explicit minimum overrides); then merge at once when every active node has
//                    contributed, else after a patience window of 1.2 x the largest round time among the
//                    active nodes within 3x of the median, clamped to [30, 300] s (60 s without timings),
//                    counted in whole seconds since the first contribution of the cycle
//   round-time EMA   0.3 old + 0.7 new over consecutive pushes 10-600 s apart
//
// The Python coordinators keep the state (contribution lists, heartbeats, profiles) and call these for
// every decision.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <set>
#include <string>
#include <vector>

#define DT_API extern "C" __attribute__((visibility("default")))

// Returns 1 (accepted, *weight_out set) or 0 (rejected, reason written, NUL-terminated, into reason[cap]).
DT_API int dts_accept_push(long long acc_version, long long push_version, int max_staleness, int n_existing,
                           const char* const* existing_nodes, const long long* existing_seq, const char* node_id,
                           long long seq, double tokens, double decay, double* weight_out, char* reason,
                           int reason_cap) {
  const long long staleness = std::max(acc_version - push_version, 0LL);
  if (staleness > max_staleness) {
    if (reason && reason_cap > 0) std::snprintf(reason, (size_t)reason_cap, "Too stale: %lld > %d", staleness, max_staleness);
    return 0;
  }
  for (int i = 0; i < n_existing; ++i) {
    if (std::strcmp(existing_nodes[i], node_id) == 0 && existing_seq[i] >= seq) {
      if (reason && reason_cap > 0)
        std::snprintf(reason, (size_t)reason_cap, "Duplicate: existing seq_num %lld >= %lld", existing_seq[i], seq);
      return 0;
    }
  }
  *weight_out = tokens * std::pow(decay, (double)staleness);
  if (reason && reason_cap > 0) reason[0] = '\0';
  return 1;
}

// active_round_times[i]: the node's expected round time if it reported one, else its observed round time,
// NaN if neither is known. Returns 1 = merge now.
DT_API int dts_should_checkpoint(int n_contribs, const char* const* contributor_nodes, int n_active,
                                 const char* const* active_nodes, const double* active_round_times,
                                 double elapsed_secs, int min_override) {
  if (n_contribs <= 0) return 0;
  int min_required;
  if (min_override > 0) min_required = min_override;
  else if (n_active <= 1) min_required = 1;
  else min_required = std::max(n_active / 2, 2);
  if (n_contribs < min_required) return 0;
  std::set<std::string> contributing;
  for (int i = 0; i < n_contribs; ++i) contributing.insert(contributor_nodes[i]);
  int active_contributed = 0;
  for (int i = 0; i < n_active; ++i) active_contributed += contributing.count(active_nodes[i]) ? 1 : 0;
  if (n_active > 0 && active_contributed >= n_active) return 1;
  std::vector<double> times;
  for (int i = 0; i < n_active; ++i)
    if (!std::isnan(active_round_times[i])) times.push_back(active_round_times[i]);
  double patience;
  if (times.empty()) {
    patience = 60.0;
  } else {
    std::sort(times.begin(), times.end());
    const double median = times[times.size() / 2];
    double cluster_max = median;
    bool any = false;
    for (double t : times)
      if (t <= median * 3.0) { cluster_max = t; any = true; }
    if (!any) cluster_max = median;
    patience = std::min(std::max(cluster_max * 1.2, 30.0), 300.0);
  }
  const double elapsed = std::floor(std::max(elapsed_secs, 0.0));  // whole seconds, as chrono num_seconds()
  return elapsed >= patience ? 1 : 0;
}

// New round time after a push at now_secs (prev NaN = none yet; last_push < 0 = first push): returns the
// updated value, or prev unchanged when the interval is outside (10, 600) s.
DT_API double dts_update_round_time(double prev, long long last_push, long long now_secs) {
  if (last_push < 0) return prev;
  const double el = (double)std::max(now_secs - last_push, 0LL);
  if (!(el > 10.0 && el < 600.0)) return prev;
  return std::isnan(prev) ? el : prev * 0.3 + el * 0.7;
}
