// ref_shim.cc — test infrastructure: a C ABI over the reference engine's own
// candidate-scoring code, compiled from its sources where they lie
// (engine/src/index/simd_distance.cc, engine/src/index/pq_codec.cc) by
// oracle/Makefile into oracle/_ref/libvectra_engine_ref.so. Only the tests
// and bench.py's CPU baseline load it, as the checker and the timed CPU
// reference of the scan path; nothing shipped calls it.
//
// The functions forward to the reference's L2SquaredDistance,
// InnerProduct, PqAdcDistance and ProductQuantizer; the exhaustive top-k
// keeps the k nearest with the reference's Neighbor / CloserFirst
// (engine/include/vectra/index/search_scratch.h:29-40) in a bounded heap as
// ShardIndex::ExhaustiveSearch does (engine/src/index/shard_index.cc:
// 110-120, 236-266).
#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

#include "vectra/index/pq_codec.h"
#include "vectra/index/search_scratch.h"
#include "vectra/index/simd_distance.h"

using vectra::index::CloserFirst;
using vectra::index::Neighbor;

extern "C" {

float ref_l2_squared_distance(const float* a, const float* b, int dim) {
  return vectra::index::L2SquaredDistance(a, b, dim);
}

float ref_inner_product(const float* a, const float* b, int dim) {
  return vectra::index::InnerProduct(a, b, dim);
}

float ref_pq_adc_distance(const float* table, const uint8_t* code, int m) {
  return vectra::index::PqAdcDistance(table, code, m);
}

// Distances from `query` to rows [n][stride]; out[n].
void ref_l2_distances(const float* query, const float* rows, int64_t n,
                      int64_t stride, int dim, float* out) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = vectra::index::L2SquaredDistance(query, rows + i * stride, dim);
}

// The k nearest of the candidates (ids, or every row when ids is null) in
// CloserFirst order; returns the count. The bounded heap restates
// PushBounded (shard_index.cc:110-120) over the reference's comparator.
int ref_exhaustive_topk(const float* query, const float* rows, int64_t n_rows,
                        int64_t stride, int dim, const uint32_t* ids,
                        int64_t n_ids, int k, float* out_d, uint32_t* out_n) {
  std::vector<Neighbor> heap;
  const size_t limit = static_cast<size_t>(k);
  auto push = [&](Neighbor c) {
    if (heap.size() < limit) {
      heap.push_back(c);
      std::push_heap(heap.begin(), heap.end(), CloserFirst());
    } else if (CloserFirst()(c, heap.front())) {
      std::pop_heap(heap.begin(), heap.end(), CloserFirst());
      heap.back() = c;
      std::push_heap(heap.begin(), heap.end(), CloserFirst());
    }
  };
  const int64_t n = ids != nullptr ? n_ids : n_rows;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t node = ids != nullptr ? ids[i] : static_cast<uint32_t>(i);
    push({vectra::index::L2SquaredDistance(query, rows + node * stride, dim),
          node});
  }
  std::sort(heap.begin(), heap.end(), CloserFirst());
  for (size_t j = 0; j < heap.size(); ++j) {
    out_d[j] = heap[j].distance;
    out_n[j] = heap[j].node;
  }
  return static_cast<int>(heap.size());
}

// The same over PQ codes [n][code_stride] with the query's table.
int ref_pq_topk(const float* table, const uint8_t* codes, int64_t n_rows,
                int64_t code_stride, int m, const uint32_t* ids, int64_t n_ids,
                int k, float* out_d, uint32_t* out_n) {
  std::vector<Neighbor> heap;
  const size_t limit = static_cast<size_t>(k);
  const int64_t n = ids != nullptr ? n_ids : n_rows;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t node = ids != nullptr ? ids[i] : static_cast<uint32_t>(i);
    const Neighbor c{
        vectra::index::PqAdcDistance(table, codes + node * code_stride, m),
        node};
    if (heap.size() < limit) {
      heap.push_back(c);
      std::push_heap(heap.begin(), heap.end(), CloserFirst());
    } else if (CloserFirst()(c, heap.front())) {
      std::pop_heap(heap.begin(), heap.end(), CloserFirst());
      heap.back() = c;
      std::push_heap(heap.begin(), heap.end(), CloserFirst());
    }
  }
  std::sort(heap.begin(), heap.end(), CloserFirst());
  for (size_t j = 0; j < heap.size(); ++j) {
    out_d[j] = heap[j].distance;
    out_n[j] = heap[j].node;
  }
  return static_cast<int>(heap.size());
}

// ProductQuantizer::FromCodebooks + ComputeDistanceTable / Encode; 0 on
// success, -1 when the reference rejects the codebooks.
int ref_pq_distance_table(int dim, int m, const float* codebooks,
                          const float* query, float* table) {
  std::string error;
  auto pq = vectra::index::ProductQuantizer::FromCodebooks(
      dim, m,
      std::vector<float>(codebooks,
                         codebooks + static_cast<size_t>(dim) *
                                         vectra::index::kPqCentroids),
      &error);
  if (!pq) return -1;
  pq->ComputeDistanceTable(query, table);
  return 0;
}

int ref_pq_encode(int dim, int m, const float* codebooks, const float* vectors,
                  int64_t n, uint8_t* codes) {
  std::string error;
  auto pq = vectra::index::ProductQuantizer::FromCodebooks(
      dim, m,
      std::vector<float>(codebooks,
                         codebooks + static_cast<size_t>(dim) *
                                         vectra::index::kPqCentroids),
      &error);
  if (!pq) return -1;
  for (int64_t i = 0; i < n; ++i) pq->Encode(vectors + i * dim, codes + i * m);
  return 0;
}

}  // extern "C"
