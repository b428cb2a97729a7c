// Multipack LPT allocator (host, C++17, pybind11).
//
// Packs documents into `n` bins (one per data-parallel rank) of capacity `c` tokens.
// For each step: take the shortest run of remaining documents whose total length reaches
// c*n, binary-search the longest prefix of that run that Longest-Processing-Time-first
// packing fits into n bins, and return the documents that land in bin `rank`.
//
// The plan must be identical on every rank and identical to the reference sampler
// (multipack_sampler.py:10-110), so the tie rules are part of the contract:
//   * feasibility check: lengths in descending order; each goes to the bin at the top of a
//     1-indexed binary min-heap, which is then sifted down preferring the right child only
//     when it is strictly smaller, and stopping when the parent is <= the chosen child;
//   * assignment: a stable ascending sort of the indices by length, visited in reverse
//     (equal lengths: the later index first); the heap carries bin ids alongside loads;
//   * binary search over prefix length m in [1, |run|] with lo = largest feasible.
// Everything here is written from that description.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <numeric>
#include <stdexcept>
#include <vector>

namespace py = pybind11;

namespace {

// Sift the root of a 1-indexed min-heap (size n) down after its load grew.
inline void sift_root(std::vector<int64_t>& load, std::vector<int64_t>* bin_id, int64_t n) {
  int64_t parent = 1;
  while (2 * parent <= n) {
    int64_t child = 2 * parent;
    if (child + 1 <= n && load[child + 1] < load[child]) child += 1;
    if (load[parent] <= load[child]) break;
    std::swap(load[parent], load[child]);
    if (bin_id) std::swap((*bin_id)[parent], (*bin_id)[child]);
    parent = child;
  }
}

// True if LPT packs `len[0..m)` into n bins of capacity c.
bool lpt_fits(const int64_t* len, int64_t m, int64_t c, int64_t n, std::vector<int64_t>& scratch,
              std::vector<int64_t>& load) {
  scratch.assign(len, len + m);
  std::sort(scratch.begin(), scratch.end(), std::greater<int64_t>());
  load.assign(n + 1, 0);
  for (int64_t x : scratch) {
    load[1] += x;
    if (load[1] > c) return false;
    sift_root(load, nullptr, n);
  }
  return true;
}

// Indices (into len[0..m)) that LPT assigns to bin `rank`, in assignment order.
std::vector<int64_t> lpt_bin(const int64_t* len, int64_t m, int64_t n, int64_t rank) {
  std::vector<int64_t> order(m);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return len[a] < len[b]; });
  std::reverse(order.begin(), order.end());
  std::vector<int64_t> load(n + 1, 0), bin_id(n + 1);
  for (int64_t i = 0; i <= n; ++i) bin_id[i] = i - 1;
  std::vector<int64_t> mine;
  for (int64_t idx : order) {
    load[1] += len[idx];
    if (bin_id[1] == rank) mine.push_back(idx);
    sift_root(load, &bin_id, n);
  }
  return mine;
}

struct StepResult {
  bool full;
  int64_t consumed;
  std::vector<int64_t> batch;
  int64_t used_tokens;
};

StepResult allocate_step(const int64_t* lengths, int64_t size, int64_t start, int64_t rank, int64_t c, int64_t n,
                         std::vector<int64_t>& scratch, std::vector<int64_t>& load) {
  int64_t total = 0, end = start;
  while (end < size) {
    total += lengths[end];
    ++end;
    if (total >= c * n) break;
  }
  const int64_t* run = lengths + start;
  const int64_t run_len = end - start;
  int64_t lo = 1, hi = 1 + run_len;
  while (hi - lo > 1) {
    int64_t mid = (lo + hi) / 2;
    if (lpt_fits(run, mid, c, n, scratch, load)) lo = mid;
    else hi = mid;
  }
  StepResult r;
  r.full = lo >= n;
  r.consumed = lo;
  r.batch = lpt_bin(run, lo, n, rank);
  for (auto& i : r.batch) i += start;
  r.used_tokens = std::accumulate(run, run + lo, int64_t(0));
  return r;
}

std::vector<int64_t> as_int64(py::array lengths) {
  py::array_t<int64_t, py::array::c_style | py::array::forcecast> arr(lengths);
  return std::vector<int64_t>(arr.data(), arr.data() + arr.size());
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "HRM-Text B200 host-native helpers (multipack LPT allocator)";

  m.def("lpt_check", [](py::array a, int64_t c, int64_t n) {
    auto v = as_int64(a);
    std::vector<int64_t> scratch, load;
    return lpt_fits(v.data(), (int64_t)v.size(), c, n, scratch, load);
  }, py::arg("lengths"), py::arg("c"), py::arg("n"));

  m.def("lpt_with_result", [](py::array a, int64_t n, int64_t rank) {
    auto v = as_int64(a);
    auto r = lpt_bin(v.data(), (int64_t)v.size(), n, rank);
    return py::array_t<int64_t>(r.size(), r.data());
  }, py::arg("lengths"), py::arg("n"), py::arg("rank"));

  m.def("allocate", [](py::array lengths, int64_t start, int64_t rank, int64_t c, int64_t n) {
    auto v = as_int64(lengths);
    std::vector<int64_t> scratch, load;
    auto r = allocate_step(v.data(), (int64_t)v.size(), start, rank, c, n, scratch, load);
    return py::make_tuple(r.full, r.consumed, py::array_t<int64_t>(r.batch.size(), r.batch.data()), r.used_tokens);
  }, py::arg("lengths"), py::arg("start_index"), py::arg("rank"), py::arg("c"), py::arg("n"));

  // Whole-epoch plan for one rank: list of index arrays plus (used, slots) token totals.
  m.def("plan_epoch", [](py::array lengths, int64_t rank, int64_t c, int64_t n, bool drop_last) {
    auto v = as_int64(lengths);
    const int64_t size = (int64_t)v.size();
    std::vector<int64_t> scratch, load;
    py::list batches;
    int64_t start = 0, used = 0, slots = 0;
    while (start < size) {
      auto r = allocate_step(v.data(), size, start, rank, c, n, scratch, load);
      start += r.consumed;
      if (!r.full) break;
      if (drop_last && start >= size) break;
      used += r.used_tokens;
      slots += n * c;
      batches.append(py::array_t<int64_t>(r.batch.size(), r.batch.data()));
    }
    return py::make_tuple(batches, used, slots);
  }, py::arg("lengths"), py::arg("rank"), py::arg("c"), py::arg("n"), py::arg("drop_last"));
}
