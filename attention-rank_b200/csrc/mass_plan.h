// Work decomposition of the attention-mass kernel, shared by the host planner and the device.
//
// For one prompt the rows of the probe are the (query head, query token) pairs of its query span.
// Rows of the query heads that share a KV head are stacked (GQA packing) into tiles of
// kMassRowTile rows, each head's tokens padded to a multiple of 8 so that every 8-row group of
// a tile belongs to one head (one TMA box). Keys are walked in 128-key tiles from the first
// span begin to the last visible key, kMassKeyTilesPerItem tiles per CTA.
#pragma once

#include "layer_kernels.h"

#if defined(__CUDACC__)
#define ARB_PLAN_FN __host__ __device__ __forceinline__
#else
#define ARB_PLAN_FN inline
#endif

namespace arb {

struct ProbeRows {
  int query_begin;  // prompt-relative, clamped to [0, length]
  int query_end;
  int padded;       // (query_end - query_begin) rounded up to a multiple of 8
};

ARB_PLAN_FN ProbeRows probe_rows(const int32_t* query_span, int length) {
  ProbeRows rows;
  int begin = query_span[0];
  int end = query_span[1];
  if (end > length) end = length;
  if (begin < 0) begin = 0;
  if (end < begin) end = begin;
  rows.query_begin = begin;
  rows.query_end = end;
  rows.padded = ((end - begin) + 7) & ~7;
  return rows;
}

ARB_PLAN_FN MassItemShape mass_item_shape(const int32_t* query_span, const int32_t* spans, int span_count,
                                          int length, int group) {
  const ProbeRows rows = probe_rows(query_span, length);
  MassItemShape shape;
  const int row_count = group * rows.padded;
  shape.row_tiles = row_count > 0 ? (row_count + kMassRowTile - 1) / kMassRowTile : 1;
  int key_lo = length;
  int key_hi = 0;
  for (int s = 0; s < span_count; ++s) {
    int b = spans[2 * s];
    int e = spans[2 * s + 1];
    if (b < 0) b = 0;
    if (e > rows.query_end) e = rows.query_end;  // keys at or past the query end are never visible
    if (e <= b) continue;
    key_lo = b < key_lo ? b : key_lo;
    key_hi = e > key_hi ? e : key_hi;
  }
  if (key_hi <= key_lo || rows.padded == 0) {
    shape.key_begin = 0;
    shape.key_tiles = 0;
    shape.key_splits = 1;
    return shape;
  }
  shape.key_begin = (key_lo / kMassKeyTile) * kMassKeyTile;
  shape.key_tiles = (key_hi - shape.key_begin + kMassKeyTile - 1) / kMassKeyTile;
  shape.key_splits = (shape.key_tiles + kMassKeyTilesPerItem - 1) / kMassKeyTilesPerItem;
  return shape;
}

ARB_PLAN_FN int mass_items_for_prompt(const MassItemShape& shape, int kv_heads) {
  return kv_heads * shape.row_tiles * shape.key_splits;
}

}  // namespace arb
