// Octet arrangement of Mode-A records (no counterpart in the reference; it feeds the lane-per-neuron
// kernels of octet.cu).
//
// Goal.  Shared-memory row d of a 4-token tile sits in bank quad d mod 8.  If the 8 records of an octet
// (8 consecutive storage positions) read, at every input position k, features of 8 distinct residues
// d mod 8, a quarter-warp's gathers and scatters are conflict-free.  That needs (1) octets whose 64
// inputs hold every residue exactly 8 times and (2) a per-record order of the 8 inputs (columns) that is
// a decomposition of the octet's record x residue multigraph into 8 perfect matchings, which exists for
// every 8-regular bipartite multigraph (Koenig's edge-colouring theorem).
//
// Step 1, group_octets_kernel (one warp per group).  Each record is summarised by its residue histogram
// (eight 4-bit counts, a 32-bit key).  Octets are filled greedily in storage order from a pool of the
// next kOcPool unplaced records (in slot order): each pick minimises sum_r (8 - have_r - h_r)^2 over the
// residues (1000 per unit of overflow), the seventh pick must leave a deficit that some unplaced record
// matches exactly, and the eighth pick is such a record, found in a hash table of the keys of all
// unplaced records of the segment (lists of records per key, in slot order).  At the benchmarked geometry
// ~91% of the octets come out exact.  Everything is deterministic (ties: lowest pool position; lists in
// slot order).  Groups are arranged in segments of at most kOcSeg records.
// Step 2, octet_columns_kernel (one thread per octet).  Column by column, a maximum matching between the
// octet's records and the residues still to be placed (residues with the most remaining inputs first,
// augmenting paths), so an exact octet gets 8 conflict-free columns; records left unmatched in a column
// take the input whose residue has the most remaining occurrences.
//
// Outputs per group (row g - g0): order[p] = the slot stored at position p (a permutation of the valid
// slots; padding slots keep their place) and kperm[p] = the input order of that record: bits 3c .. 3c+2
// give the original input index k placed in column c.  Both depend only on the indices.
#include "common.cuh"

namespace gl {

constexpr int kOcHash = 8192;   // hash slots: >= the 6435 possible residue histograms of 8 inputs
constexpr int kOcPool = 256;    // pool of candidate records per pick
constexpr int kOcSeg = 32768;   // records arranged together (multiple of 8; list positions fit 16 bits)
constexpr uint32_t kOcEmpty = 0xFFFFFFFFu;

__host__ __device__ constexpr int32_t oc_identity_perm() {
  return (0 << 0) | (1 << 3) | (2 << 6) | (3 << 9) | (4 << 12) | (5 << 15) | (6 << 18) | (7 << 21);
}

struct OcSmem {
  uint32_t key[kOcHash];       // residue histogram of the slot's records (kOcEmpty: free)
  uint32_t pe[kOcHash];        // list cursor (low 16 bits) and list end (high 16 bits) in `lst`
  uint32_t used[kOcSeg / 32];  // records already placed
  int pool_n[kOcPool];         // pool: segment-local record, its key
  uint32_t pool_k[kOcPool];
};

__device__ __forceinline__ uint32_t oc_key(const int16_t* __restrict__ rec, int dmax) {
  const Rec8 r = load_rec8(rec, dmax);
  uint32_t v = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) v += 1u << (4 * (r.i[k] & 7));
  return v;
}

__device__ __forceinline__ uint32_t oc_hash(uint32_t key) { return (key * 2654435761u) >> 19; }

__device__ __forceinline__ int oc_find(const OcSmem& s, uint32_t key) {
  uint32_t h = oc_hash(key);
  for (int i = 0; i < kOcHash; ++i) {
    const uint32_t k = s.key[h];
    if (k == key) return (int)h;
    if (k == kOcEmpty) return -1;
    h = (h + 1) & (kOcHash - 1);
  }
  return -1;
}

__device__ __forceinline__ bool oc_used(const OcSmem& s, int n) { return (s.used[n >> 5] >> (n & 31)) & 1u; }

// First unplaced record with key slot h other than `excl`, or -1; advances the slot's cursor past
// placed records (benign when several lanes do it: they only skip placed entries).
__device__ int oc_first(OcSmem& s, const int32_t* __restrict__ lst, int m, int h, int excl) {
  const uint32_t pe = s.pe[h];
  int p = (int)(pe & 0xFFFFu);
  const int e = (int)(pe >> 16);
  while (p < e && (unsigned)lst[p] < (unsigned)m && oc_used(s, lst[p])) ++p;
  if (p != (int)(pe & 0xFFFFu)) s.pe[h] = (uint32_t)p | ((uint32_t)e << 16);
  for (int q = p; q < e; ++q) {
    const int n = lst[q];
    if ((unsigned)n < (unsigned)m && !oc_used(s, n) && n != excl) return n;
  }
  return -1;
}

__global__ void __launch_bounds__(32) group_octets_kernel(const int16_t* __restrict__ idx,
                                                          const int32_t* __restrict__ counts, int D, int64_t NB,
                                                          int64_t g0, int64_t g1, int32_t* __restrict__ order,
                                                          int32_t* __restrict__ kperm) {
  extern __shared__ __align__(16) unsigned char oc_raw[];
  OcSmem& s = *reinterpret_cast<OcSmem*>(oc_raw);
  const int lane = threadIdx.x;
  const int64_t g = g0 + blockIdx.x;
  const int slots = (int)(NB * 8);
  const int ng = min(max(__ldg(counts + g), 0), slots);
  const int16_t* gidx = idx + g * (int64_t)slots * 8;
  int32_t* gord = order + (g - g0) * (int64_t)slots;
  int32_t* gkp = kperm + (g - g0) * (int64_t)slots;  // scratch for the key lists until octet_columns_kernel
  for (int p = ng + lane; p < slots; p += 32) gord[p] = p;
  for (int s0 = 0; s0 < ng; s0 += kOcSeg) {
    const int m = min(kOcSeg, ng - s0);
    int32_t* lst = gkp + s0;
    for (int i = lane; i < kOcHash; i += 32) {
      s.key[i] = kOcEmpty;
      s.pe[i] = 0;
    }
    for (int i = lane; i < kOcSeg / 32; i += 32) s.used[i] = 0;
    __syncwarp();
    // 1. count the records of every key
    for (int n = lane; n < m; n += 32) {
      const uint32_t k = oc_key(gidx + (int64_t)(s0 + n) * 8, D - 1);
      uint32_t h = oc_hash(k);
      for (int probe = 0; probe < kOcHash; ++probe) {  // the table never fills: at most 6435 distinct keys
        const uint32_t prev = atomicCAS(&s.key[h], kOcEmpty, k);
        if (prev == kOcEmpty || prev == k) break;
        h = (h + 1) & (kOcHash - 1);
      }
      atomicAdd(&s.pe[h], 1u << 16);
    }
    __syncwarp();
    // 2. list ranges: exclusive prefix sum of the counts over the slots (lane L owns 256 slots)
    constexpr int per = kOcHash / 32;
    int tot = 0;
    for (int i = 0; i < per; ++i) tot += (int)(s.pe[lane * per + i] >> 16);
    int incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(kFullMask, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - tot;
    __syncwarp();
    for (int i = 0; i < per; ++i) {
      const int h = lane * per + i;
      const int c = (int)(s.pe[h] >> 16);
      s.pe[h] = (uint32_t)run | ((uint32_t)(run + c) << 16);
      run += c;
    }
    __syncwarp();
    // 3. fill the lists in slot order (batches of 32 records; equal keys ordered by lane)
    for (int b0 = 0; b0 < m; b0 += 32) {
      const int n = b0 + lane;
      const bool act = n < m;
      const unsigned am = __ballot_sync(kFullMask, act);
      if (act) {
        const int h = oc_find(s, oc_key(gidx + (int64_t)(s0 + n) * 8, D - 1));
        const unsigned mm = __match_any_sync(am, h);
        const int leader = __ffs(mm) - 1;
        const int rank = __popc(mm & ((1u << lane) - 1));
        int base = 0;
        if (lane == leader) base = (int)(atomicAdd(&s.pe[h], (unsigned)__popc(mm)) & 0xFFFFu);
        base = __shfl_sync(mm, base, leader);
        if (base + rank < m) lst[base + rank] = n;
      }
      __syncwarp();
    }
    // cursors back to the list starts: the start of slot h is the end of slot h - 1
    {
      uint32_t st[per];
      for (int i = 0; i < per; ++i) {
        const int h = lane * per + i;
        st[i] = h == 0 ? 0u : (s.pe[h - 1] >> 16);
      }
      __syncwarp();
      for (int i = 0; i < per; ++i) {
        const int h = lane * per + i;
        s.pe[h] = st[i] | (s.pe[h] & 0xFFFF0000u);
      }
    }
    __threadfence_block();
    __syncwarp();
    // 4. the pool: the first records in slot order
    int psize = min(m, kOcPool), next = psize;
    for (int i = lane; i < psize; i += 32) {
      s.pool_n[i] = i;
      s.pool_k[i] = oc_key(gidx + (int64_t)(s0 + i) * 8, D - 1);
    }
    __syncwarp();
    // 5. fill octets
    int placed = 0;
    while (placed < m) {
      uint64_t have = 0;  // 8-bit count per residue
      const int on = min(8, m - placed);
      for (int j = 0; j < on; ++j) {
        int take = -1, tpool = -1;
        uint32_t tkey = 0;
        if (j == 7) {  // an exact complement among all unplaced records
          uint32_t need = 0;
          bool ok = true;
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int c = (int)((have >> (8 * r)) & 255);
            if (c > 8) ok = false;
            else need |= (uint32_t)(8 - c) << (4 * r);
          }
          if (ok) {
            const int h = oc_find(s, need);
            int t = -1;
            if (h >= 0 && lane == 0) t = oc_first(s, lst, m, h, -1);
            take = __shfl_sync(kFullMask, t, 0);
            tkey = need;
          }
          __syncwarp();
        }
        if (take < 0 && psize <= 0) {  // cannot happen (the pool holds every unplaced record below `next`)
          placed = m;
          break;
        }
        if (take < 0) {
          int best = 0x7fffffff, bi = 0x7fffffff;
          for (int i = lane; i < psize; i += 32) {
            const uint32_t k = s.pool_k[i];
            int sc = 0;
            uint32_t need = 0;
            bool ok = true;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              const int d = 8 - (int)((have >> (8 * r)) & 255) - (int)((k >> (4 * r)) & 15);
              sc += d < 0 ? -1000 * d : d * d;
              if (d < 0) ok = false;
              else need |= (uint32_t)d << (4 * r);
            }
            if (j == 6 && sc < 1000 && on == 8) {
              const int h = ok ? oc_find(s, need) : -1;
              if (h < 0 || oc_first(s, lst, m, h, s.pool_n[i]) < 0) sc += 500;
            }
            if (sc < best) {
              best = sc;
              bi = i;
            }
          }
#pragma unroll
          for (int off = 16; off; off >>= 1) {
            const int ob = __shfl_xor_sync(kFullMask, best, off);
            const int oi = __shfl_xor_sync(kFullMask, bi, off);
            if (ob < best || (ob == best && oi < bi)) {
              best = ob;
              bi = oi;
            }
          }
          tpool = bi;
          take = s.pool_n[bi];
          tkey = s.pool_k[bi];
        } else if (take < next) {  // the complement is a pool member: find its position
          for (int i0 = 0; i0 < psize && tpool < 0; i0 += 32) {
            const int i = i0 + lane;
            const unsigned hit = __ballot_sync(kFullMask, i < psize && s.pool_n[i] == take);
            if (hit) tpool = i0 + __ffs(hit) - 1;
          }
        }
        __syncwarp();
        if (lane == 0) {
          s.used[take >> 5] |= 1u << (take & 31);
          gord[s0 + placed] = s0 + take;
        }
        __syncwarp();
        if (tpool >= 0) {  // refill the pool position with the next unplaced record in slot order
          while (next < m && oc_used(s, next)) ++next;
          if (lane == 0) {
            if (next < m) {
              s.pool_n[tpool] = next;
              s.pool_k[tpool] = oc_key(gidx + (int64_t)(s0 + next) * 8, D - 1);
            } else {
              s.pool_n[tpool] = s.pool_n[psize - 1];
              s.pool_k[tpool] = s.pool_k[psize - 1];
            }
          }
          if (next < m) ++next;
          else --psize;
          __syncwarp();
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) have += (uint64_t)((tkey >> (4 * r)) & 15) << (8 * r);
        ++placed;
      }
    }
    __syncwarp();
  }
}

// Step 2: the column order of each octet's inputs.
__global__ void __launch_bounds__(128) octet_columns_kernel(const int16_t* __restrict__ idx,
                                                            const int32_t* __restrict__ counts, int D, int64_t NB,
                                                            int64_t g0, int64_t g1, const int32_t* __restrict__ order,
                                                            int32_t* __restrict__ kperm) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t g = g0 + tid / NB;
  if (g >= g1) return;
  const int o = (int)(tid % NB);
  const int slots = (int)(NB * 8);
  const int ng = min(max(__ldg(counts + g), 0), slots);
  const int64_t row = (g - g0) * (int64_t)slots;
  const int base = 8 * o;
  const int m = min(max(ng - base, 0), 8);
  unsigned char res[8][8];
  int avail[8], perm[8];
  for (int a = 0; a < 8; ++a) {
    perm[a] = 0;
    avail[a] = a < m ? 0xFF : 0;
    if (a < m) {
      const int slot = min(max(__ldg(order + row + base + a), 0), slots - 1);
      const Rec8 r = load_rec8(idx + (g * (int64_t)slots + slot) * 8, D - 1);
      for (int k = 0; k < 8; ++k) res[a][k] = (unsigned char)(r.i[k] & 7);
    }
  }
  for (int c = 0; c < 8 && m > 0; ++c) {
    int rcount[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int rmask[8];
    for (int a = 0; a < m; ++a) {
      rmask[a] = 0;
      for (int k = 0; k < 8; ++k)
        if (avail[a] >> k & 1) {
          rcount[res[a][k]]++;
          rmask[a] |= 1 << res[a][k];
        }
    }
    int ord[8];
    for (int r = 0; r < 8; ++r) ord[r] = r;
    for (int i = 0; i < 8; ++i)  // residues by decreasing remaining count (stable)
      for (int j = 7; j > i; --j)
        if (rcount[ord[j]] > rcount[ord[j - 1]]) {
          const int t = ord[j];
          ord[j] = ord[j - 1];
          ord[j - 1] = t;
        }
    int matchN[8];
    for (int a = 0; a < 8; ++a) matchN[a] = -1;
    for (int oi = 0; oi < 8; ++oi) {
      const int r0 = ord[oi];
      if (rcount[r0] == 0) continue;
      int prevN[8], prevR[8], qr[8], qh = 0, qt = 0, endN = -1;
      bool visN[8];
      for (int a = 0; a < 8; ++a) {
        prevN[a] = -1;
        prevR[a] = -2;
        visN[a] = false;
      }
      qr[qt++] = r0;
      prevR[r0] = -1;
      while (qh < qt && endN < 0) {
        const int r = qr[qh++];
        for (int a = 0; a < m && endN < 0; ++a) {
          if (visN[a] || !(rmask[a] >> r & 1)) continue;
          visN[a] = true;
          prevN[a] = r;
          if (matchN[a] < 0) endN = a;
          else if (prevR[matchN[a]] == -2 && qt < 8) {
            prevR[matchN[a]] = a;
            qr[qt++] = matchN[a];
          }
        }
      }
      if (endN >= 0) {  // augment along the path back to r0
        int a = endN;
        for (int guard = 0; guard < 16; ++guard) {
          const int r = prevN[a];
          const int pa = prevR[r];
          matchN[a] = r;
          if (pa < 0) break;
          a = pa;
        }
      }
    }
    for (int a = 0; a < m; ++a) {
      int r = matchN[a];
      int kk = -1;
      if (r >= 0) {
        for (int k = 0; k < 8 && kk < 0; ++k)
          if ((avail[a] >> k & 1) && res[a][k] == r) kk = k;
      }
      if (kk < 0) {  // unmatched: the input whose residue remains most often
        for (int k = 0; k < 8; ++k)
          if ((avail[a] >> k & 1) && (kk < 0 || rcount[res[a][k]] > rcount[res[a][kk]])) kk = k;
      }
      avail[a] &= ~(1 << kk);
      rcount[res[a][kk]]--;
      perm[a] |= kk << (3 * c);
    }
  }
  for (int a = 0; a < 8; ++a)
    if (base + a < slots) kperm[row + base + a] = a < m ? perm[a] : oc_identity_perm();
}

}  // namespace gl

using namespace gl;

extern "C" int gl_group_octets(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0,
                               int64_t g1, int32_t* order, int32_t* kperm, void* stream) {
  if (D < 1 || D > 32767 || NB < 1 || g0 < 0 || g1 < g0) return GL_ERR_SHAPE;
  if (NB * 8 > 2147483647LL) return GL_ERR_SHAPE;
  if (g1 == g0) return GL_OK;
  if (!idx || !counts || !order || !kperm) return GL_ERR_NULL;
  if ((uintptr_t)idx & 15) return GL_ERR_ALIGN;
  if (g1 - g0 > 2147483647LL) return GL_ERR_SHAPE;
  const size_t smem = sizeof(OcSmem);
  int rc = ensure_dynamic_smem((const void*)group_octets_kernel, smem);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  group_octets_kernel<<<(unsigned)(g1 - g0), 32, smem, st>>>(idx, counts, (int)D, NB, g0, g1, order, kperm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  const int64_t threads = (g1 - g0) * NB;
  const int64_t blocks = (threads + 127) / 128;
  if (blocks > 2147483647LL) return GL_ERR_SHAPE;
  octet_columns_kernel<<<(unsigned)blocks, 128, 0, st>>>(idx, counts, (int)D, NB, g0, g1, order, kperm);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(2);
  return GL_OK;
}
