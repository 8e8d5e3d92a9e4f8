// Tile-record helpers shared by the LoRA kernels that walk the tile records.
//
// A tile record is {tile, first segment, segment count, slot of the first segment}:
// one per 128-token row tile holding segment tokens.  Segments are sorted by start
// and do not overlap; these helpers clamp every index to the segment table, so a
// malformed record reads as fewer rows (and is reported) instead of reading past
// the table.
#pragma once

#include "lf_common.cuh"

namespace lf {
namespace rec {

constexpr int kTile = LF_TILE_TOKENS;

__device__ __forceinline__ bool aborted(const int32_t* flag) {
  return *reinterpret_cast<const volatile int32_t*>(flag) != 0;
}

// Number of sub-items (segments) of a record, clamped to the segment table.
__device__ __forceinline__ int sub_items(const int4& rec, int n_segs) {
  int k = rec.z < 1 ? 1 : rec.z;
  if (rec.y >= 0 && rec.y < n_segs && k > n_segs - rec.y) k = n_segs - rec.y;
  return k;
}

// Slot of sub-item j (the record carries the first one); -1 reads zeros by TMA fill.
__device__ __forceinline__ int32_t sub_slot(const int4& rec, int j, const int32_t* seg_slot, int n_segs) {
  if (j == 0) return rec.w;
  const int g = rec.y + j;
  return (g >= 0 && g < n_segs) ? __ldg(seg_slot + g) : -1;
}

// Tile rows [lo, hi) that one segment covers (lo == hi: none).
struct SubRows {
  int lo, hi;
};

__device__ __forceinline__ SubRows clip_rows(int64_t s0, int64_t l0, int64_t row0, int64_t n_tokens) {
  const int64_t lo = max(s0, row0) - row0;
  const int64_t hi = min(min(s0 + l0, row0 + kTile), n_tokens) - row0;
  if (hi <= lo) return {0, 0};
  return {int(lo), int(hi)};
}

// {start, len, slot} of the record's first segment (slot -1 if out of range).
__device__ __forceinline__ int4 first_seg(const int4& rec, const int32_t* seg_start, const int32_t* seg_len,
                                          const int32_t* seg_slot, int n_segs) {
  if (rec.y < 0 || rec.y >= n_segs) return make_int4(0, 0, -1, 0);
  return make_int4(__ldg(seg_start + rec.y), __ldg(seg_len + rec.y), __ldg(seg_slot + rec.y), 0);
}

// Rows of sub-item j of a record; seg0 is the record's first segment, loaded
// ahead of time.  A segment whose slot is out of range, or a first segment
// whose slot disagrees with the record, covers no rows and is reported.
__device__ __forceinline__ SubRows rows_of(const int4& rec, int j, const int4& seg0, int64_t row0,
                                           int64_t n_tokens, const int32_t* seg_start, const int32_t* seg_len,
                                           const int32_t* seg_slot, int n_segs, int n_slots, int32_t* status,
                                           bool report) {
  int4 sg = seg0;
  if (j > 0) {
    const int g = rec.y + j;
    if (g < 0 || g >= n_segs) {
      if (report) set_status(status, LF_STATUS_BAD_SEGMENT);
      return {0, 0};
    }
    sg = make_int4(__ldg(seg_start + g), __ldg(seg_len + g), __ldg(seg_slot + g), 0);
  } else if (rec.y < 0 || rec.y >= n_segs || sg.z != rec.w) {
    if (report) set_status(status, LF_STATUS_BAD_SEGMENT);
    return {0, 0};
  }
  if (sg.z < 0 || sg.z >= n_slots) {
    if (report) set_status(status, LF_STATUS_BAD_SLOT);
    return {0, 0};
  }
  return clip_rows(sg.x, sg.y, row0, n_tokens);
}

}  // namespace rec
}  // namespace lf
