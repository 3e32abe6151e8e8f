// Host-side cell orderings that the sampler attaches to every batch
// (headwater/src/sampler.rs:655-784). The attention kernels run in the
// permuted token order these produce: column attention under col_perm, the
// feature (outbound) and neighbor (inbound) masks under the two reverse
// Cuthill-McKee orders, so that related cells land in the same 128-token tiles
// and the tile plan stays sparse.
//
// Both orderings are total orders (ties end on the cell position), so any
// correct sort reproduces the reference's result bit for bit. Samples are
// independent and are spread over host threads.
#include <algorithm>
#include <cstdint>
#include <deque>
#include <exception>
#include <numeric>
#include <thread>
#include <vector>

namespace rt {
namespace order {

// Cells sorted by (padding last, column id, position): sampler.rs:655-668.
void column_order(const int32_t* col, const uint8_t* pad, int S, uint16_t* out) {
  std::vector<uint16_t> idx(S);
  std::iota(idx.begin(), idx.end(), 0);
  std::sort(idx.begin(), idx.end(), [&](uint16_t a, uint16_t b) {
    if (pad[a] != pad[b]) return pad[a] < pad[b];
    if (col[a] != col[b]) return col[a] < col[b];
    return a < b;
  });
  std::copy(idx.begin(), idx.end(), out);
}

// Reverse Cuthill-McKee order of the sample's rows over the FK graph, then
// cells sorted by (padding last, row rank, position): sampler.rs:672-784.
// Row graph: i -> j for fk_adj[i][j] (outbound, the feature mask's graph) or
// fk_adj[j][i] (inbound), self loops dropped, neighbours in ascending index.
// Each BFS starts at the first unvisited row of least degree among the rows
// that hold a non-padding cell, or at the first unvisited row when none is
// left; neighbours are queued in a stable order of ascending degree; the
// visit order is reversed. Cells whose row id is >= R rank last.
void rcm_order(const uint8_t* fk, const uint16_t* rows, const uint8_t* pad, int S, int R, bool outbound,
               uint16_t* out) {
  std::vector<std::vector<int>> adj(R);
  for (int i = 0; i < R; ++i)
    for (int j = 0; j < R; ++j)
      if (i != j && (outbound ? fk[(size_t)i * R + j] : fk[(size_t)j * R + i]) == 1) adj[i].push_back(j);
  std::vector<char> used(R, 0), seen(R, 0);
  for (int p = 0; p < S; ++p)
    if (pad[p] == 0 && rows[p] < R) used[rows[p]] = 1;
  std::vector<int> visit;
  visit.reserve(R);
  std::deque<int> queue;
  std::vector<int> nb;
  while ((int)visit.size() < R) {
    int start = -1;
    for (int i = 0; i < R; ++i)
      if (!seen[i] && used[i] && (start < 0 || adj[i].size() < adj[start].size())) start = i;
    if (start < 0)
      for (int i = 0; i < R && start < 0; ++i)
        if (!seen[i]) start = i;
    if (start < 0) break;
    seen[start] = 1;
    queue.push_back(start);
    while (!queue.empty()) {
      const int node = queue.front();
      queue.pop_front();
      visit.push_back(node);
      nb.clear();
      for (int n : adj[node])
        if (!seen[n]) nb.push_back(n);
      std::stable_sort(nb.begin(), nb.end(), [&](int a, int b) { return adj[a].size() < adj[b].size(); });
      for (int n : nb)
        if (!seen[n]) {
          seen[n] = 1;
          queue.push_back(n);
        }
    }
  }
  std::reverse(visit.begin(), visit.end());
  for (int i = 0; i < R; ++i)
    if (!seen[i]) visit.push_back(i);
  std::vector<int64_t> rank(R, 0);
  for (size_t k = 0; k < visit.size(); ++k) rank[visit[k]] = (int64_t)k;
  std::vector<int64_t> cell_rank(S);
  for (int p = 0; p < S; ++p) cell_rank[p] = rows[p] < R ? rank[rows[p]] : INT64_MAX;
  std::vector<uint16_t> idx(S);
  std::iota(idx.begin(), idx.end(), 0);
  std::sort(idx.begin(), idx.end(), [&](uint16_t a, uint16_t b) {
    if (pad[a] != pad[b]) return pad[a] < pad[b];
    if (cell_rank[a] != cell_rank[b]) return cell_rank[a] < cell_rank[b];
    return a < b;
  });
  std::copy(idx.begin(), idx.end(), out);
}

// Runs fn(b) for every sample on up to hardware_concurrency threads; returns
// false if any sample threw (allocation failure).
template <class F>
bool for_each_sample(int batch, F fn) {
  const int n = std::max(1, std::min<int>(batch, (int)std::thread::hardware_concurrency()));
  std::vector<char> failed(n, 0);
  auto work = [&](int t) {
    try {
      for (int b = t; b < batch; b += n) fn(b);
    } catch (const std::exception&) {
      failed[t] = 1;
    }
  };
  if (n == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < n; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
  }
  return std::find(failed.begin(), failed.end(), 1) == failed.end();
}

}  // namespace order
}  // namespace rt

extern "C" int rt_column_order(const int32_t* column_ids, const uint8_t* is_padding, int32_t batch,
                               int32_t seq_len, uint16_t* perm) {
  if (batch < 0 || seq_len < 0 || seq_len > 65536) return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return RT_OK;
  if (!column_ids || !is_padding || !perm) return RT_ERR_INVALID_ARGUMENT;
  const bool ok = rt::order::for_each_sample(batch, [&](int b) {
    const size_t o = (size_t)b * seq_len;
    rt::order::column_order(column_ids + o, is_padding + o, seq_len, perm + o);
  });
  return ok ? RT_OK : RT_ERR_WORKSPACE;
}

extern "C" int rt_rcm_order(const uint8_t* fk_adj, const uint16_t* seq_row_ids, const uint8_t* is_padding,
                            int32_t batch, int32_t seq_len, int32_t max_rows, int32_t outbound, uint16_t* perm) {
  if (batch < 0 || seq_len < 0 || seq_len > 65536 || max_rows < 0 || max_rows > 65536)
    return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return RT_OK;
  if (!seq_row_ids || !is_padding || !perm || (max_rows > 0 && !fk_adj)) return RT_ERR_INVALID_ARGUMENT;
  const bool ok = rt::order::for_each_sample(batch, [&](int b) {
    const size_t o = (size_t)b * seq_len;
    rt::order::rcm_order(fk_adj + (size_t)b * max_rows * max_rows, seq_row_ids + o, is_padding + o, seq_len,
                         max_rows, outbound != 0, perm + o);
  });
  return ok ? RT_OK : RT_ERR_WORKSPACE;
}
