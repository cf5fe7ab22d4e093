// Fixed partition of the absolute key axis shared by the decode-attention kernels (attention.cu,
// attention_tc.cu) and their combine kernel.
#pragma once

namespace q38 {

constexpr int CH = 128;      // keys per chunk (fixed absolute chunks)

// Key groups: the absolute key axis is cut into 128-key chunks and the chunks into groups by a
// fixed partition - one chunk per group for the first 64 chunks (8,192 keys), four per group up
// to chunk 512 (65,536 keys), eight beyond - so short contexts keep many CTAs while long ones
// write few partials.  The partition depends on key positions only, never on how many rows run.
constexpr int G_T0 = 64, G_T1 = 512;           // tier boundaries in chunks
__host__ __device__ __forceinline__ int groups_for(int nchunks) {
  if (nchunks <= G_T0) return nchunks;
  if (nchunks <= G_T1) return G_T0 + (nchunks - G_T0 + 3) / 4;
  return G_T0 + (G_T1 - G_T0) / 4 + (nchunks - G_T1 + 7) / 8;
}
__host__ __device__ __forceinline__ int group_first_chunk(int grp) {
  if (grp < G_T0) return grp;
  if (grp < G_T0 + (G_T1 - G_T0) / 4) return G_T0 + 4 * (grp - G_T0);
  return G_T1 + 8 * (grp - G_T0 - (G_T1 - G_T0) / 4);
}
__host__ __device__ __forceinline__ int group_chunks(int grp) {
  return grp < G_T0 ? 1 : (grp < G_T0 + (G_T1 - G_T0) / 4 ? 4 : 8);
}

}  // namespace q38
