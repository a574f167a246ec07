// Expert-parallel transport over peer memory: the destination functor of the
// fused quantise + dispatch kernel, and the launch interfaces of ep_p2p.cu.
//
// Every rank holds one receive buffer of the same layout, mapped into every
// peer's address space (NVLink P2P; torch symmetric memory on the Python
// side).  Byte offsets inside it are identical on all ranks:
//   flags  int32 [world]            barrier epochs, one slot per sender
//   counts int32 [world, E]         row s = sender s's routed rows per expert
//   xq     int8  [cap, H]           received token rows, grouped by local expert
//   xs     fp32  [cap]              their scales
//   src    int32 [cap]              return address: sender * tk_max + flat slot
//   yhome  bf16  [tk_max, H]        results of this rank's own slots, by flat slot
//   dup    int32 [cap]              (deduplicated dispatch) for each received row the
//                                   position of the same token's first row on this
//                                   rank, whose bytes it copies, or -1 if it was sent
// No TMA and no multicast touch peer memory: plain stores only.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace w4a8 {

// Destinations of token t's quantised row for the expert-parallel dispatch:
// slot j goes to the receive buffer of the rank owning its expert, at the row
// reserved for it by the counts exchange (dest_base) plus its rank among this
// sender's slots of that expert (inv_pos - offsets, from this rank's align).
struct PeerRows {
  const int32_t* ids;        // [T*topk] global expert of every slot
  int topk, E, epr, rank;
  int64_t tk_max;            // slots per rank at most: encodes return addresses
  int H;
  const int32_t* offsets;    // [E+1] this rank's align of its slots by global expert
  const int32_t* inv_pos;    // [T*topk] sorted position of every slot
  const int32_t* dest_base;  // [E] first receive row for this rank's slots of e on e's owner (-1: none)
  uint8_t* const* peers;     // [world] receive-buffer bases as seen from this GPU
  int64_t xq_off, xs_off, src_off;
  int32_t* home_pos;         // [T*topk] out: the slot's own index once dispatched, -1 if dropped
  int64_t dup_off = -1;      // >= 0: a token's row crosses to each rank once (see dup above)
  __device__ __forceinline__ int count() const { return topk; }
  __device__ __forceinline__ int8_t* row(int t, int d, float scale, bool meta) const {
    const int64_t f = static_cast<int64_t>(t) * topk + d;
    const int e = ids[f];
    const int base = (e >= 0 && e < E) ? dest_base[e] : -1;
    if (base < 0) {
      if (meta) home_pos[f] = -1;
      return nullptr;
    }
    const int64_t pos = static_cast<int64_t>(base) + (inv_pos[f] - offsets[e]);
    const int owner = e / epr;
    uint8_t* b = peers[owner];
    // deduplicated: the row position of this token's first slot on the same
    // remote rank (rows for this rank itself are all written here: a local
    // copy later would read and write them again)
    int64_t prim = -1;
    if (dup_off >= 0 && owner != rank) {
      for (int d2 = 0; d2 < d; ++d2) {
        const int64_t f2 = static_cast<int64_t>(t) * topk + d2;
        const int e2 = ids[f2];
        if (e2 < 0 || e2 >= E || e2 / epr != owner) continue;
        const int b2 = dest_base[e2];
        if (b2 < 0) continue;
        prim = static_cast<int64_t>(b2) + (inv_pos[f2] - offsets[e2]);
        break;
      }
    }
    if (meta) {
      reinterpret_cast<float*>(b + xs_off)[pos] = scale;
      reinterpret_cast<int32_t*>(b + src_off)[pos] = static_cast<int32_t>(rank * tk_max + f);
      if (dup_off >= 0) reinterpret_cast<int32_t*>(b + dup_off)[pos] = static_cast<int32_t>(prim);
      home_pos[f] = static_cast<int32_t>(f);
    }
    if (prim >= 0) return nullptr;   // the owner copies the bytes from the token's first row there
    return reinterpret_cast<int8_t*>(b + xq_off) + pos * H;
  }
};

cudaError_t launch_ep_dispatch(const __nv_bfloat16* x, int64_t x_stride0, int T, int H, const PeerRows& dest,
                               cudaStream_t stream);

}  // namespace w4a8
