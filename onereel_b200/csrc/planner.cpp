// Native per-request planner: scene layout key frames, the work-balanced partition (paper Algorithm 1), the K/V
// exchange sets and the Eq. 2 path choice — src/onereel/parallel/comm.py:18-112 and src/onereel/layout.py:54-78 of
// the reference, restated in C++ with the same float64 arithmetic so that every cut is bit-identical:
//   - work prefix sums are sequential double additions (numpy's cumsum),
//   - the boundary search is "first index with W[i] >= x" (numpy searchsorted side='left') with
//     x = p * (W / n) - 1e-12 * W,
//   - the in-scene offset is rounded half-to-even (Python's round) with nearbyint in the default rounding mode,
//   - a zero search index wraps to the last element, as Python's W[i - 1] does for i = 0.
#include <algorithm>
#include <cfenv>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <set>
#include <utility>
#include <vector>

#include "orl_common.h"

namespace orl {
namespace {

constexpr double kCLin = 0.02581842, kCAtt = 6.753627e-07, kEffScene = 1.0;   // comm.py:15

struct Layout {
  std::vector<int> lengths;
  int halo = 0;
  int sides = 0;                          // 0 adj, 1 prev, 2 next
  std::vector<std::vector<int>> extra;    // per scene, as given (unsorted)
  std::vector<int> start;                 // first frame per scene, plus the total

  int n() const { return static_cast<int>(lengths.size()); }
  int frames() const { return start.back(); }

  std::vector<int> halo_frames(int j) const {
    std::vector<int> out;
    if (halo == 0) return out;
    if (j > 0 && sides != 2)
      for (int f = std::max(start[j - 1], start[j] - halo); f < start[j]; ++f) out.push_back(f);
    if (j + 1 < n() && sides != 1)
      for (int f = start[j + 1]; f < std::min(start[j + 2], start[j + 1] + halo); ++f) out.push_back(f);
    return out;
  }
  std::vector<int> shared_frames(int j) const {
    std::vector<int> out = halo_frames(j);
    std::vector<int> ex = extra[j];
    std::sort(ex.begin(), ex.end());
    for (int f : ex) {
      if (f >= start[j] && f < start[j + 1]) continue;
      if (std::find(out.begin(), out.end(), f) != out.end()) continue;
      out.push_back(f);
    }
    return out;
  }
  std::vector<int> key_frames(int j) const {
    std::vector<int> out;
    for (int f = start[j]; f < start[j + 1]; ++f) out.push_back(f);
    auto s = shared_frames(j);
    out.insert(out.end(), s.begin(), s.end());
    return out;
  }
};

bool make_layout(const orl_layout* in, Layout* L) {
  if (in == nullptr || in->n_scenes <= 0 || in->lengths == nullptr || in->halo < 0 || in->sides < 0 || in->sides > 2)
    return false;
  L->lengths.assign(in->lengths, in->lengths + in->n_scenes);
  L->halo = in->halo;
  L->sides = in->sides;
  L->start.assign(1, 0);
  for (int v : L->lengths) {
    if (v <= 0) return false;
    L->start.push_back(L->start.back() + v);
  }
  L->extra.assign(in->n_scenes, {});
  if (in->extra_offsets != nullptr) {
    for (int j = 0; j < in->n_scenes; ++j) {
      const int a = in->extra_offsets[j], b = in->extra_offsets[j + 1];
      if (a < 0 || b < a || (b > a && in->extra_frames == nullptr)) return false;
      L->extra[j].assign(in->extra_frames + a, in->extra_frames + b);
    }
  }
  return true;
}

using Interval = std::pair<long long, long long>;

std::vector<Interval> frame_tokens(const std::vector<int>& frames, long long T) {
  std::vector<Interval> out;   // runs of consecutive frames in list order, as token intervals
  for (int f : frames) {
    if (!out.empty() && out.back().second == f * T) out.back().second = (f + 1LL) * T;
    else out.push_back({f * T, (f + 1LL) * T});
  }
  return out;
}

std::vector<Interval> merge(std::vector<Interval> iv) {
  std::vector<Interval> out;
  iv.erase(std::remove_if(iv.begin(), iv.end(), [](const Interval& x) { return x.first >= x.second; }), iv.end());
  std::sort(iv.begin(), iv.end());
  for (auto& x : iv) {
    if (!out.empty() && x.first <= out.back().second) out.back().second = std::max(out.back().second, x.second);
    else out.push_back(x);
  }
  return out;
}

std::vector<double> query_cost(const Layout& L, long long T, const int32_t* text, long long extra_keys) {
  std::vector<double> c(L.n());
  for (int j = 0; j < L.n(); ++j) {
    const long long keys = static_cast<long long>(L.key_frames(j).size()) * T + (text ? text[j] : 0) + extra_keys;
    c[j] = kCLin + kCAtt * kEffScene * static_cast<double>(keys);
  }
  return c;
}

// comm.py:25-40; bounds[0..n] cuts
bool balanced(const std::vector<long long>& sizes, const std::vector<double>& cost, int n, std::vector<long long>* b) {
  const int m = static_cast<int>(sizes.size());
  long long L = 0;
  for (long long s : sizes) L += s;
  if (L < n || n < 1) return false;
  std::vector<long long> a(m + 1, 0);
  std::vector<double> W(m + 1, 0.0);
  for (int j = 0; j < m; ++j) {
    a[j + 1] = a[j] + sizes[j];
    W[j + 1] = W[j] + static_cast<double>(sizes[j]) * cost[j];
  }
  const double target = W[m] / n;
  b->assign(1, 0);
  const int saved = std::fegetround();
  std::fesetround(FE_TONEAREST);
  for (int p = 1; p < n; ++p) {
    const double x = p * target - 1e-12 * W[m];
    const int i = static_cast<int>(std::lower_bound(W.begin(), W.end(), x) - W.begin());
    const int im1 = i - 1 >= 0 ? i - 1 : m;          // Python's index -1 wraps to the last element
    const int cm1 = i - 1 >= 0 ? i - 1 : m - 1;
    const long long r = static_cast<long long>(std::nearbyint((p * target - W[im1]) / cost[cm1]));
    b->push_back(std::min(std::max(a[im1] + r, b->back() + 1), L - (n - p)));
  }
  std::fesetround(saved);
  b->push_back(L);
  return true;
}

}  // namespace
}  // namespace orl

using namespace orl;

extern "C" int orl_key_frames(const orl_layout* layout, int scene, int32_t* frames, int capacity) {
  Layout L;
  if (!make_layout(layout, &L) || scene < 0 || scene >= L.n()) return ORL_ERR_ARG;
  auto kf = L.key_frames(scene);
  if (frames == nullptr || capacity < static_cast<int>(kf.size())) return -static_cast<int>(kf.size()) - 1000;
  std::copy(kf.begin(), kf.end(), frames);
  return static_cast<int>(kf.size());
}

extern "C" int orl_query_cost(const orl_layout* layout, long long T, const int32_t* text, long long extra_keys,
                              double* cost) {
  Layout L;
  if (!make_layout(layout, &L) || T <= 0 || cost == nullptr) return ORL_ERR_ARG;
  auto c = query_cost(L, T, text, extra_keys);
  std::copy(c.begin(), c.end(), cost);
  return ORL_OK;
}

extern "C" int orl_balanced(const int64_t* sizes, const double* cost, int n_scenes, int n, int64_t* bounds) {
  if (sizes == nullptr || cost == nullptr || bounds == nullptr || n_scenes <= 0 || n <= 0) return ORL_ERR_ARG;
  std::vector<long long> s(sizes, sizes + n_scenes), b;
  std::vector<double> c(cost, cost + n_scenes);
  if (!balanced(s, c, n, &b)) return ORL_ERR_ARG;
  std::copy(b.begin(), b.end(), bounds);
  return ORL_OK;
}

extern "C" int orl_partition(const orl_layout* layout, long long T, int n, int mode, const int32_t* text,
                             long long extra_keys, int granularity, int64_t* bounds) {
  Layout L;
  if (!make_layout(layout, &L) || T <= 0 || n <= 0 || bounds == nullptr) return ORL_ERR_ARG;
  const long long tokens = L.frames() * T;
  if (mode == ORL_MODE_ULYSSES || n == 1 || granularity == ORL_GRAN_TOKENS) {
    if ((mode == ORL_MODE_ULYSSES || n == 1) && tokens % n != 0) return ORL_ERR_ARG;
    for (int r = 0; r <= n; ++r) bounds[r] = r * tokens / n;
    return ORL_OK;
  }
  std::vector<long long> sizes;
  for (int v : L.lengths) sizes.push_back(static_cast<long long>(v) * T);
  std::vector<long long> own;
  if (!balanced(sizes, query_cost(L, T, text, extra_keys), n, &own)) return ORL_ERR_ARG;
  if (granularity == ORL_GRAN_SCENES) {
    // comm.py:53-62: each balanced boundary moved to the nearest scene start that keeps every rank non-empty
    if (L.n() < n) return ORL_ERR_ARG;
    std::vector<long long> starts;
    for (int s : L.start) starts.push_back(s * T);
    std::vector<long long> b(1, 0);
    for (int p = 1; p < n; ++p) {
      long long best = -1, best_d = 0;
      for (int idx = 1; idx + 1 < static_cast<int>(starts.size()); ++idx) {
        const long long s = starts[idx];
        if (!(s > b.back() && idx <= L.n() - (n - p))) continue;
        const long long d = std::llabs(s - own[p]);
        if (best < 0 || d < best_d) best = s, best_d = d;
      }
      if (best < 0) return ORL_ERR_ARG;
      b.push_back(best);
    }
    b.push_back(tokens);
    std::copy(b.begin(), b.end(), bounds);
    return ORL_OK;
  }
  if (granularity != ORL_GRAN_BALANCED) return ORL_ERR_ARG;
  std::copy(own.begin(), own.end(), bounds);
  return ORL_OK;
}

extern "C" int orl_needed(const orl_layout* layout, long long T, long long own_lo, long long own_hi,
                          const int32_t* extra, int n_extra, int64_t* intervals, int capacity) {
  Layout L;
  if (!make_layout(layout, &L) || T <= 0 || own_lo > own_hi || (n_extra > 0 && extra == nullptr)) return ORL_ERR_ARG;
  std::vector<int> ex(extra, extra + std::max(n_extra, 0));
  std::sort(ex.begin(), ex.end());
  std::vector<Interval> iv = frame_tokens(ex, T);
  for (int j = 0; j < L.n(); ++j) {
    const long long lo = L.start[j] * T, hi = L.start[j + 1] * T;
    if (lo < own_hi && hi > own_lo) {
      iv.push_back({lo, hi});
      auto s = frame_tokens(L.shared_frames(j), T);
      iv.insert(iv.end(), s.begin(), s.end());
    }
  }
  std::vector<Interval> out;
  for (auto& x : merge(iv)) {
    const Interval left{x.first, std::min(x.second, own_lo)}, right{std::max(x.first, own_hi), x.second};
    if (left.first < left.second) out.push_back(left);
    if (right.first < right.second) out.push_back(right);
  }
  const int n = static_cast<int>(out.size());
  if (intervals == nullptr || capacity < n) return -n - 1000;
  for (int i = 0; i < n; ++i) {
    intervals[2 * i] = out[i].first;
    intervals[2 * i + 1] = out[i].second;
  }
  return n;
}

extern "C" int orl_choose_path(const orl_layout* layout, long long T, const int64_t* bounds, int n, double theta,
                               const int32_t* extra, int n_extra, orl_path* path) {
  Layout L;
  if (!make_layout(layout, &L) || T <= 0 || n <= 0 || bounds == nullptr || path == nullptr) return ORL_ERR_ARG;
  long long remote = 0;
  for (int r = 0; r < n; ++r) {
    const int need = -orl_needed(layout, T, bounds[r], bounds[r + 1], extra, n_extra, nullptr, 0) - 1000;
    std::vector<int64_t> iv(2 * std::max(need, 1));
    const int got = orl_needed(layout, T, bounds[r], bounds[r + 1], extra, n_extra, iv.data(), need);
    if (got < 0) return ORL_ERR_ARG;
    long long rows = 0;
    for (int i = 0; i < got; ++i) rows += iv[2 * i + 1] - iv[2 * i];
    remote = std::max(remote, rows);
  }
  const long long tokens = L.frames() * T;
  path->remote_rows = remote;
  path->V_G = 2.0 * static_cast<double>(remote);
  path->V_U = 4.0 * static_cast<double>(tokens) * (n - 1) / (static_cast<double>(n) * n);
  path->gather = path->V_G < theta * path->V_U ? 1 : 0;
  return ORL_OK;
}
