/*
 * granule_b200.h — C ABI of the B200 (sm_100a) sparse-pooling kernels.
 *
 * The reference exposes this hot path only as a Python protocol between
 * Level1Runtime and its backend objects, on top of Triton launches:
 *   forward : sparse_pooling/autograd.py:213-233  (Level1Runtime.forward)
 *             -> kernels/ops.py:104-154 fused_forward_states
 *                (Triton fwd_pool_kernel, kernels/triton_fused.py:289-358)
 *             -> kernels/ops.py:182-199 merge_finalize (mean: pre = s / n_g)
 *   backward: sparse_pooling/autograd.py:236-300  (Level1Runtime.backward / _triton_backward)
 *             -> kernels/ops.py:242-249 dense_coefficients (mean: c1 = g_pre / n_g)
 *             -> kernels/ops.py:265-278 launch_dense_backward
 *                (Triton bwd_dense_kernel, kernels/triton_fused.py:402-472)
 *   optimizer: sparse_pooling/optim.py:26-64 _adamw_kernel, launched by FusedAdamW.step (optim.py:91-126)
 * and its native library's ctypes ABI follows the same conventions this header
 * keeps (sparse_pooling/kernels/cuda/abi.cu:9-62, sparse_pool.cu:12-44,
 * backends/cuda/runtime.py:34-121): plain pointers and sizes, caller-owned
 * memory, an explicit stream, a version query, and negative status codes
 * instead of exceptions.
 *
 * Conventions
 *   - Every entry point returns GL_OK (0) or a negative GlStatus; it never
 *     throws and never exits.  gl_status_string() names a status.
 *   - All buffers are caller-owned device memory.  No entry point allocates
 *     device memory.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default) of the
 *     current device; calls return before the GPU finishes.
 *   - Parameters use the reference's Mode-A storage unchanged
 *     (sparse_pooling/layout.py:5-8, 123-140), C = 8 neurons per block, fan-in 8:
 *       idx  [G_total, NB, 8, 8] int16, w [G_total, NB, 8, 8] f32, b [G_total, NB, 8] f32
 *     Neuron slot s of group g has flat index f = g*NB*8 + s; its record is
 *     idx[8f .. 8f+7], w[8f .. 8f+7], b[f].  Slots s >= counts[g] are padding
 *     and are masked out of every sum.
 *   - Sharding: a call processes the contiguous group range [g0, g1) and reads
 *     its pooled columns at y/gpre column (g - g0).
 */
#ifndef GRANULE_B200_H
#define GRANULE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GL_ABI_VERSION 17

typedef enum GlStatus {
  GL_OK = 0,
  GL_ERR_NULL = -1,          /* a required pointer is NULL */
  GL_ERR_SHAPE = -2,         /* inconsistent sizes (B, D, NB, group range, strides) */
  GL_ERR_ALIGN = -3,         /* a pointer is not aligned for vector access */
  GL_ERR_UNSUPPORTED = -4,   /* pool/activation/tile combination not built */
  GL_ERR_SMEM = -5,          /* the tile does not fit in shared memory */
  GL_ERR_LAUNCH = -6,        /* the CUDA launch failed (see gl_last_cuda_error) */
  GL_ERR_DEVICE = -7,        /* no usable device / attribute query failed */
  GL_ERR_CAPACITY = -8       /* the problem is larger than an allocation-free entry point's fixed scratch */
} GlStatus;

/* Pool ids: the reference's operators (sparse_pooling/config.py:22-29) and the "sum"
   extension.  Activation ids follow config.py:33.  With a = act(z) over the valid slots of a
   group (n of them):
     MEAN     pre = sum a / n                          SUM  pre = sum a
     MAX      pre = max a; its winner is the smallest slot attaining the maximum
              (kernels/triton_fused.py:129-140); backward: gl_bwd_events_f32
     LME      pre = tau * (log sum e^(a/tau) - log n); param = log2(e) / tau;
              stat = L2 = log2 sum 2^(a * param)        (pytorch_reference.py:80-85)
     POWER    pre = (sum a^p / n)^(1/p), a = relu(z) >= 0; param = p >= 1   (:86-92)
     SOFTMAX  pre = sum a e^(beta a) / sum e^(beta a); param = log2(e) * beta;
              stat = L2 = log2 sum 2^(a * param)        (:93-98)
     TOPK     pre = sum of act(z) over the k slots with the largest z (ties: the smaller slot)
              / min(k, n); k a power of two <= 64; `winners` [B, ldwin >= (g1-g0) k] receives
              the slots, largest first, -1 past min(k, n) (:66-77); backward:
              gl_bwd_events_f32 with k events per (token, group)
   The smooth pools' backward is gl_bwd_f32 / gl_bwd_shared_f32 with the reference's
   per-(token, group) coefficients (kernels/ops.py:242-262): dz = c1 * h * act'(z) with
     MEAN/SUM h = 1 (c1 = gpre / n for MEAN, computed by the kernel; gpre for SUM)
     LME      h = 2^(a * param - c2)                  c1 = gpre, c2 = L2
     POWER    h = (a * c2)^(p - 1), 0 where z <= 0    c1 = gpre / n (0 where pre = 0), c2 = 1 / pre
     SOFTMAX  h = 2^(a * param - c2) (1 + beta (a - c3)), beta = param * ln 2
                                                      c1 = gpre, c2 = L2, c3 = pre */
enum { GL_POOL_MEAN = 0, GL_POOL_SUM = 1, GL_POOL_MAX = 2, GL_POOL_LME = 3, GL_POOL_POWER = 4, GL_POOL_SOFTMAX = 5,
       GL_POOL_TOPK = 6 };
enum { GL_ACT_IDENTITY = 0, GL_ACT_RELU = 1, GL_ACT_GELU = 2 };
/* Storage types of parameters (the reference's default layer dtype is bfloat16); the kernels
   compute in fp32 and write fp32 gradients. */
enum { GL_DTYPE_F32 = 0, GL_DTYPE_BF16 = 1 };

/* Forward: pre[t, g - g0] = pool_{valid s of g} act(z[t, g, s]),
 *   z[t, g, s] = b[f] + sum_k w[8f+k] * x[t, idx[8f+k]],
 * pool = one of the pool ids above.  `pre` is written, not accumulated.
 * Replaces fused_forward_states + merge_finalize (kernels/ops.py:104-199). */
typedef struct GlFwdArgs {
  const float* x;           /* [B, ldx] token-major input, D used columns */
  const int16_t* idx;       /* Mode-A indices (see conventions), values in [0, D) */
  const float* w;           /* weights */
  const float* b;           /* bias */
  const int32_t* counts;    /* [G_total] valid neurons per group */
  float* pre;               /* [B, ldp] pooled output, columns 0 .. g1-g0-1 */
  int64_t B, D, NB;         /* tokens, input features, blocks per group */
  int64_t g0, g1;           /* group range processed by this call */
  int64_t ldx, ldp;         /* row strides in elements */
  int32_t pool;             /* GL_POOL_* */
  int32_t act;              /* GL_ACT_* */
  int32_t tokens;           /* token tile (0 = automatic; else 1, 2, 4 or 8) */
  int32_t groups_per_cta;   /* groups per thread block (0 = automatic) */
  float* wabsmax;           /* optional [g1-g0] output: max |w| over each group's valid slots
                               (the backward's fixed-point bound); NULL = not computed */
  const int32_t* order;     /* optional [g1-g0, NB*8] processing order (gl_group_order): position p of
                               group g processes slot order[g-g0][p]; NULL = slot order */
  const int16_t* lidx;      /* optional input locality (gl_group_feature_map): the records as positions */
  const int16_t* fmap;      /*   in their group's feature list fmap [g1-g0, fcap], nfeat [g1-g0] entries */
  const int32_t* nfeat;     /*   each; a block then stages only its group's features.  NULL = off */
  int64_t fcap;             /* row length of fmap (>= max nfeat) */
  int32_t* winners;         /* GL_POOL_MAX: optional [B, ldwin] output, the winning slot of each (t, g) */
  int64_t ldwin;
  float* stat;              /* GL_POOL_LME / SOFTMAX: optional [B, ldstat] output, the log2-normaliser L2 */
  int64_t ldstat;
  float param;              /* the pool's parameter (see the pool ids); unused otherwise */
  int32_t k;                /* GL_POOL_TOPK: the number of slots kept; unused otherwise */
  int32_t wdtype;           /* storage type of w and b: GL_DTYPE_F32 or GL_DTYPE_BF16 */
  int32_t reserved3;        /* 0 */
} GlFwdArgs;

/* Backward: with c1[t, g] = gpre[t, g - g0] / counts[g] (mean) or gpre (the other pools) and
 *   dz[t, f] = c1[t, g] * h * act'(z[t, f]) for valid slots (0 for padding; h as for the pool ids):
 *   dx[t, d]   += sum_{f, k: idx[8f+k] = d} dz[t, f] * w[8f+k]
 *   dw[8f + k] += sum_t dz[t, f] * x[t, idx[8f+k]]
 *   db[f]      += sum_t dz[t, f]
 * dx, dw and db are accumulated (+=); dw/db use the weight/bias layout, so they
 * can be the reference's FP32 `main_grad` buffers (autograd.py:357-363).
 * With `wabsmax` and `rowmax` (both from the calls below, or the forward's
 * wabsmax output) the block-private dX tile is accumulated in int32 fixed point
 * (faster); with both NULL it is accumulated with fp32 atomics.  Non-finite
 * coefficients or weights make the affected tokens' dx non-finite, as fp32
 * arithmetic would.
 * Replaces dense_coefficients + launch_dense_backward (kernels/ops.py:242-278). */
typedef struct GlBwdArgs {
  const float* x;
  const int16_t* idx;
  const float* w;
  const float* b;
  const int32_t* counts;
  const float* gpre;        /* [B, ldg] dL/dpre, columns 0 .. g1-g0-1 */
  float* dx;                /* [B, lddx] fp32, accumulated */
  float* dw;                /* weight-shaped fp32, accumulated */
  float* db;                /* bias-shaped fp32, accumulated */
  int64_t B, D, NB;
  int64_t g0, g1;
  int64_t ldx, ldg, lddx;
  int32_t pool;
  int32_t act;
  int32_t tokens;           /* token tile (0 = automatic; else 1, 2, 4 or 8) */
  int32_t groups_per_cta;   /* 0 = automatic */
  const float* wabsmax;     /* [g1-g0] max |w| per group (gl_group_absmax_f32), or NULL */
  const int32_t* rowmax;    /* [g1-g0] max records per input feature (gl_group_index_maxcount), or NULL */
  const int32_t* order;     /* optional processing order, as in GlFwdArgs */
  const int16_t* lidx;      /* optional input locality, as in GlFwdArgs */
  const int16_t* fmap;
  const int32_t* nfeat;
  int64_t fcap;
  const float* c2;          /* smooth pools: [B, ldg] coefficients c2, c3 (see the pool ids); else NULL */
  const float* c3;
  float param;              /* the pool's parameter */
  int32_t wdtype;           /* storage type of w and b (dw, db, dx stay fp32) */
} GlBwdArgs;

/* Adam(W) step over n elements, in place (sparse_pooling/optim.py:26-64), in fp32 arithmetic:
 *   m = b1 m + (1-b1) g ;  v = b2 v + (1-b2) g^2
 *   p = p (1 - lr wd) - lr (m / bc1) / (sqrt(v / bc2) + eps)
 *   g = 0 when zero_grad != 0 (the reference's fused zero_grad).
 * bc1 = 1 - b1^t and bc2 = 1 - b2^t are passed in, as the reference does.  The gradient g is fp32;
 * p is fp32 or bf16 (pdtype), m and v fp32 or bf16 (mdtype, stored round-to-nearest-even).  With
 * `master` (fp32, bf16 parameters) the update runs on the master copy and p receives it rounded to
 * nearest; without one a bf16 p is rounded stochastically when `stochastic` is set (uniform noise
 * below the bf16 ulp from a counter-based hash of (seed, element), then truncation, optim.py:55-62),
 * else to nearest. */
typedef struct GlAdamArgs {
  void* p;
  float* g;
  void* m;
  void* v;
  int64_t n;
  float lr, beta1, beta2, eps, weight_decay, bc1, bc2;
  int32_t zero_grad;
  float* master;            /* optional fp32 master weights of a bf16 p; NULL = none */
  int32_t pdtype;           /* GL_DTYPE_* of p */
  int32_t mdtype;           /* GL_DTYPE_* of m and v */
  int32_t stochastic;       /* bf16 p without master: 1 = stochastic rounding, 0 = nearest */
  uint32_t seed;            /* stochastic rounding stream */
} GlAdamArgs;

int gl_abi_version(void);
const char* gl_status_string(int status);
/* Last CUDA error code seen by a failed launch on this thread (0 if none). */
int gl_last_cuda_error(void);

int gl_fwd_f32(const GlFwdArgs* args, void* stream);
int gl_bwd_f32(const GlBwdArgs* args, void* stream);
int gl_adam_f32(const GlAdamArgs* args, void* stream);

/* Per-group bounds of the fixed-point backward (no counterpart in the reference):
 *   gl_group_absmax_f32:     out[g-g0] = max |w[8f+k]| over the valid slots f of group g
 *   gl_group_index_maxcount: out[g-g0] = max over features d of the number of valid
 *                            (slot, k) records of group g with idx == d
 * The second depends only on the indices; callers compute it once per layer. */
int gl_group_absmax_f32(const float* w, const int32_t* counts, int64_t NB, int64_t g0, int64_t g1, float* out,
                        void* stream);
int gl_group_index_maxcount(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0,
                            int64_t g1, int32_t* out, void* stream);

/* Per-group input feature maps (no counterpart in the reference): nf[g-g0] = number of distinct
 * features read by group g's valid records; with fmap (row length cap) also the sorted list
 * fmap[g-g0][0 .. nf-1], and with lidx (indices-shaped) the records as positions in that list.
 * Call once with fmap = lidx = NULL to size cap = max nf.  Depends only on the indices. */
int gl_group_feature_map(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0, int64_t g1,
                         int32_t cap, int32_t* nf, int16_t* fmap, int16_t* lidx, void* stream);

/* Bank-aware processing order (no counterpart in the reference): out[g-g0][p], p < NB*8, is a
 * permutation of group g's slots (valid slots first, padding slots in place) such that the
 * `unit` consecutive positions served by one shared-memory wavefront read rows in distinct bank
 * groups (row d mod unit) for as many of their 8 inputs as possible.  unit = 32 / token tile:
 * 4 for the forward's tile of 8, 8 for the backward's tile of 4; 4 and 8 are supported, and
 * unit = 48 builds units of 8 (scored mod 8) whose halves are also scored mod 4, serving both.
 * Depends only on the indices; callers compute it once per layer. */
int gl_group_order(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0, int64_t g1,
                   int32_t unit, int32_t* out, void* stream);

/* Octet arrangement of Mode-A storage (no counterpart in the reference), for the lane-per-neuron kernels
 * below: out order[g-g0][p] (p < NB*8) = the slot stored at position p, a permutation of group g's valid
 * slots (padding slots keep their place), chosen so that every 8 consecutive positions ("octet") hold
 * records whose 64 inputs cover each residue d mod 8 as evenly as possible; kperm[g-g0][p] = that record's
 * input order: bits 3c .. 3c+2 are the original input index k placed in column c, chosen so that at each
 * column the octet's 8 records read 8 distinct residues where the octet allows it.  A caller stores
 * idx / w (and their gradients) as rec'[p][c] = rec[order[p]][k_c] and b as b'[p] = b[order[p]].  Depends
 * only on the indices; callers compute it once per layer.  kperm doubles as the kernel's scratch until it
 * is written. */
int gl_group_octets(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0, int64_t g1,
                    int32_t* order, int32_t* kperm, void* stream);

/* Lane-per-neuron forward / backward (no counterpart in the reference; the sums of gl_fwd_f32 /
 * gl_bwd_f32 for the mean and sum pools, fp32 parameters, any activation), tuned for octet-arranged
 * storage and correct on any storage order.  One lane per record, a warp step = 4 octets: the forward
 * stages 8 tokens as two 4-token half tiles, the backward 4 tokens and an int32 dX tile at one fixed-point
 * scale per token for the block's groups (`wabsmax`, `rowmax` required; K = min(2^22, 0.9 2^31 / sum of
 * the block's rowmax)), so D <= (shared memory per block - 1 KiB) / 32 (7,232 on B200; GL_ERR_SMEM beyond).
 * `tokens` must be 0 (or 8 / 4); order, locality, winners and stat must be NULL; other pools and bf16
 * storage return GL_ERR_UNSUPPORTED.  dx, dw, db are accumulated as in gl_bwd_f32; the forward writes pre
 * (and wabsmax when given) as gl_fwd_f32 does.  w and dw use the octet weight layout: within a group, each
 * block of 32 consecutive records (slot counts are multiples of 32) stores the records' weights 0-3 (16
 * bytes each, record j at byte 16 j) and then their weights 4-7 (at byte 512 + 16 j); idx and b keep the
 * record layout. */
int gl_fwd_octet_f32(const GlFwdArgs* args, void* stream);
int gl_bwd_octet_f32(const GlBwdArgs* args, void* stream);
/* The same backward with `feat_prefix` from gl_group_feature_prefix over the args' group range g0 .. g1: the
 * int32 dX tile then accumulates the rounding's raw bits and its flush subtracts the magic number's bit pattern
 * once per record input of the feature in the block's groups, one instruction fewer per shared atomic; dx, dw,
 * db as gl_bwd_octet_f32 (dX bit for bit: integer sums modulo 2^32).  feat_prefix must describe the current
 * indices and counts. */
int gl_bwd_octet_prefix_f32(const GlBwdArgs* args, const int32_t* feat_prefix, void* stream);
/* out [(g1-g0+1) * D] int32: out[i*D + d] = number of (record, input) pairs of groups g0 .. g0+i-1 (their valid
 * records) whose index, clamped to D-1, is d.  Mode-A indices [G, NB, 8, 8] int16 (any storage order). */
int gl_group_feature_prefix(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0, int64_t g1,
                            int32_t* out, void* stream);

/* Mode B (shared index records), fp32.  Block j of group g holds C neurons (C = 8, 16, 32 or 64)
 * sharing one 8-input record; slot s = j*C + c is valid iff s < counts[g]:
 *   z[t, g, j, c] = b[g][j][c] + sum_k w[g][j][c][k] * x[t, idx[g][j][k]]
 * Storage is the reference's (sparse_pooling/layout.py:20-33, 123-179), canonical
 *   idx [G, NB, 8] int16, w [G, NB, C, 8] f32, b [G, NB, C] f32,
 * or fragment-packed (packed != 0), read in place.  Forward writes pre[t, g - g0] as
 * gl_fwd_f32 does; backward accumulates dx, dw, db (dw/db in the storage layout) as gl_bwd_f32
 * does, with fp32 shared-memory reductions.
 * Replaces the reference's Mode-B CUDA kernels (kernels/cuda/sparse_pool_fwd.cuh:311,
 * sparse_pool_bwd.cuh:387-876; entries sparse_pool.cu:12-44) for fp32 parameters. */
typedef struct GlSharedArgs {
  const float* x;           /* [B, ldx] */
  const int16_t* idx;       /* 16-byte aligned */
  const float* w;           /* 16-byte aligned */
  const float* b;           /* 16-byte aligned */
  const int32_t* counts;    /* [G_total] */
  float* pre;               /* forward: [B, ldp] */
  const float* gpre;        /* backward: [B, ldg] dL/dpre */
  float* dx;                /* backward: [B, lddx], accumulated */
  float* dw;                /* backward: weight-shaped, accumulated, 16-byte aligned */
  float* db;                /* backward: bias-shaped, accumulated, 16-byte aligned */
  int64_t B, D, NB, C;      /* tokens, input features, blocks per group, neurons per block */
  int64_t g0, g1;
  int64_t ldx, ldp, ldg, lddx;
  int32_t pool;             /* GL_POOL_* */
  int32_t act;              /* GL_ACT_* */
  int32_t packed;           /* 0 = canonical storage, 1 = fragment-packed */
  int32_t tokens;           /* token tile (0 = automatic; else 1, 2, 4 or 8) */
  int32_t groups_per_cta;   /* 0 = automatic */
  int32_t wdtype;           /* storage type of w and b (dw, db, dx stay fp32) */
  int32_t* winners;         /* forward, GL_POOL_MAX: optional [B, ldwin] winning slots */
  int64_t ldwin;
  float* stat;              /* forward, GL_POOL_LME / SOFTMAX: optional [B, ldstat] L2 output */
  int64_t ldstat;
  const float* c2;          /* backward, smooth pools: [B, ldg] coefficients c2, c3 */
  const float* c3;
  float param;              /* the pool's parameter */
  int32_t k;                /* forward, GL_POOL_TOPK: the number of slots kept */
} GlSharedArgs;

int gl_fwd_shared_f32(const GlSharedArgs* args, void* stream);
/* Mode B with bf16 parameters on the tensor cores (fragment-packed storage, wdtype = GL_DTYPE_BF16),
 * the reference's bf16 arithmetic (its layers cast x to the layer dtype, sparse_pooling/autograd.py:349-354,
 * and run m16n8k8 BF16 tiles with fp32 accumulation, kernels/cuda/sparse_pool_fwd.cuh:311): x is rounded
 * to bf16 (nearest even) as it is staged, every product bf16 x bf16 is exact, sums are fp32.
 * Forward: pools MEAN, SUM and MAX (winners optional, smallest slot on ties), any activation; `tokens`
 * = 0 (automatic) or 16, 32, 64.  Other configurations return GL_ERR_UNSUPPORTED. */
int gl_fwd_shared_tc(const GlSharedArgs* args, void* stream);
/* Backward of the mean and sum pools on the same path, the reference's default "split" gradient precision
 * (kernels/cuda/sparse_pool_bwd.cuh:387-876): dz = c1 act'(z) is carried as hi + lo bf16 (16 significant
 * bits), so dz * w and dz * x are summed in fp32 from exact products; dx, dw, db (fp32, dw / db in the
 * packed layout) are accumulated as gl_bwd_shared_f32 does.  `tokens` = 0 (automatic), 16 or 32; the
 * x slab and a 4-byte dX tile share the shared memory, so D is bounded (GL_ERR_SMEM beyond).
 * With `wabsmax` ([g1-g0] max |w| over each group's valid slots) and `rowmax` ([g1-g0] the largest number
 * of valid record inputs of the group on one feature) the dX tile is accumulated in int32 fixed point at
 * a power-of-two scale per (token, group) with m C |c1| max|w| max|act'| scale <= 2^30 (faster; a token
 * whose bound is not finite gets NaN); with both NULL it is accumulated with fp32 atomics. */
int gl_bwd_shared_tc(const GlSharedArgs* args, const float* wabsmax, const int32_t* rowmax, void* stream);
/* The same backward for layers with input-supergroup connectivity (supergroups.py), one CTA per token
 * tile and chunk of buckets of one input set (replaces the reference's grouped sg_dx / sg_dw kernels,
 * kernels/cuda/sparse_pool_sg.cuh).  Every record of bucket (q, g, first unit, units) reads only the S
 * features feat[q], so a CTA stages only those rows and a dX tile of S rows, with a larger token tile
 * (`tokens` 0 = automatic, 32, 64 or 128).  Buckets of groups outside [g0, g1) are skipped.  With rowmax
 * ([n] the bucket's largest number of record inputs on one feature) and wabsmax ([g1-g0] max |w| per
 * group) the dX tile is int32 fixed point at one power-of-two scale per token and chunk; with both NULL
 * it is fp32. */
typedef struct GlSetArgs {
  const int16_t* feat;      /* [Q, S] sorted features of each input set */
  const int32_t* buckets;   /* [n, 4] int32 (q, g, first unit, units), units of the layout's unit_blocks */
  const int32_t* chunks;    /* [nchunks, 3] (q, first bucket, end bucket): buckets of set q, at most
                               max_chunk of them */
  const int32_t* rowmax;    /* optional [n] */
  const float* wabsmax;     /* optional [g1-g0] */
  int64_t S, nchunks, max_chunk;  /* max_chunk <= 256 */
} GlSetArgs;
int gl_bwd_shared_tc_sets(const GlSharedArgs* args, const GlSetArgs* sets, void* stream);
/* Forward of the mean and sum pools on the same chunks (replaces the reference's grouped sg_fwd): pre is
 * zeroed (NaN for the mean of a group without valid slots), then every (token, bucket) partial, divided by
 * the group's count for the mean, is added with one fp32 atomic, so the sum order is not fixed. */
int gl_fwd_shared_tc_sets(const GlSharedArgs* args, const GlSetArgs* sets, void* stream);
/* Token tile the tensor-core forward (backward = 0) or backward (1) would use for input_dim D, or a
 * negative status (GL_ERR_SMEM when D does not fit). */
int gl_shared_tc_auto_tokens(int64_t D, int32_t backward);
int gl_bwd_shared_f32(const GlSharedArgs* args, void* stream);
/* Token tile the automatic choice would use for input_dim D, or a negative status. */
int gl_shared_auto_tokens(int64_t D, int32_t backward);

/* Deterministic Mode-B backward (PhysicalPlan.reduction = "deterministic"; replaces the reference's
 * deterministic reductions, kernels/cuda/sg_det.cu): the same sums as gl_bwd_shared_f32 for the
 * mean / sum pools, bitwise repeatable.  dW / db have one owner per record that adds the token tiles
 * in order; dX is accumulated exactly in 64-bit integers: every (token, record, k) sum is rounded to
 * an integer at the power-of-two scale qscale[t] and added to dxq, a caller-zeroed int64 [B, D]
 * (row stride D) buffer, and a second kernel adds dxq[t, d] * qinv[t] to dx.  The caller picks
 * qscale[t] = 2^e_t with sum_d |dx[t, d]| * 2^e_t < 2^61 (a bound: sum_g |c1[t, g]| * n_g * 8 *
 * max|w|_g * max|act'| * 2^e_t <= 2^60), qinv[t] = 2^-e_t (NaN for a token whose bound is not
 * finite, which makes its dx NaN). */
int gl_bwd_shared_det_f32(const GlSharedArgs* args, int64_t* dxq, const float* qscale, const float* qinv,
                          void* stream);

/* Allocation-free deterministic Mode-B backward (no counterpart in the reference): the same
 * computation and results as gl_bwd_shared_det_f32, for callers that cannot allocate device memory
 * where the backward runs (a plugin whose host framework owns all device memory through its own
 * pool, or a loop that cannot afford cudaMalloc's possible device synchronisation).  The int64 dX
 * scratch lives in a fixed array inside the library instead of a caller buffer, so B * D must be at
 * most GL_DET_STATIC_MAX_ELEMS (8 MiB of int64; larger problems return GL_ERR_CAPACITY); every
 * device that loads the library holds that array until exit.  Each call checks all its arguments
 * before it touches the array, looks up the array's device address in the calling thread's current
 * context (the first call in a context may load the library's device code: make it before any stream
 * capture), and clears the entries it uses on `stream`.  All calls on one device share the array:
 * calls whose GPU work can overlap race on it.  Calls no cudaMalloc, cudaFree or allocating library
 * routine. */
#define GL_DET_STATIC_MAX_ELEMS (1 << 20)
int gl_bwd_shared_det_static_f32(const GlSharedArgs* args, const float* qscale, const float* qinv, void* stream);

/* Winner-event backward of max and top-K pooling, Mode A or Mode B (replaces
 * kernels/triton_fused.py:476-520 bwd_events_kernel, launched by kernels/ops.py:281-293).  For each
 * (t, g, j) in [0, B) x [g0, g1) x [0, kev), with s = winners[t, (g-g0) kev + j] (a slot the
 * forward's max or top-K chose) and c = coef[t, g-g0] (dL/dpre, divided by min(k, n) for top-K):
 *   dz = c * act'(z[t, g, s]); db[s] += dz; dw[s][k] += dz * x[t, idx_k]; dx[t, idx_k] += dz * w[s][k]
 * Events with s < 0 or c == 0 are skipped.  Storage as in GlBwdArgs (Mode A) or GlSharedArgs (Mode B:
 * shared = 1, C, packed); dx, dw, db are accumulated. */
typedef struct GlEventArgs {
  const float* x;           /* [B, ldx] */
  const int16_t* idx;       /* 16-byte aligned */
  const float* w;           /* 16-byte aligned */
  const float* b;
  const int32_t* winners;   /* [B, ldwin] */
  const float* coef;        /* [B, ldc] */
  float* dx;                /* [B, lddx] */
  float* dw;                /* 8-byte aligned */
  float* db;
  int64_t B, D, NB, C;      /* C: neurons per block (Mode B) */
  int64_t g0, g1;
  int64_t ldx, ldwin, ldc, lddx;
  int32_t shared;           /* 0 = Mode A, 1 = Mode B */
  int32_t packed;           /* Mode B storage: 0 = canonical, 1 = fragment-packed */
  int32_t act;              /* GL_ACT_* */
  int32_t kev;              /* events per (token, group): 1 (max; 0 reads as 1) or the top-K k */
  int32_t wdtype;           /* storage type of w and b */
  int32_t reserved;         /* 0 */
} GlEventArgs;

int gl_bwd_events_f32(const GlEventArgs* args, void* stream);

/* Compact K16/C16 execution of the Cover-TopK/16 layer, fp32.
 * Replaces the reference's kgen entry points at K = 16 (experimental/kgen/kgen_abi.cu,
 * kernels kgen.cuh:142-536), called by KgenFunction (experimental/kgen_layer.py:61-143) with
 * the layer's lowered storage (experimental/kgen_lowered.py:147-201):
 *   w [G, NB16, 16, 16] f32, b [G, NB16, 16] f32, record f = g*NB16 + j; neuron slot 16 j + n
 *   of output g is valid iff it is < counts[g];
 *   feat [Q, S] int16: the input features of set q;
 *   env [G*NB16, 16] uint8: record f reads x[:, feat[q][env[f, k]]], q = its bucket's set;
 *   buckets [nb, 4] int32 (q, g, first record j, records), sorted by q; q_off [Q+1] int32: the
 *   bucket range of set q; rec_off [nb+1] int32: exclusive prefix sum of buckets[:, 3].
 * Forward:  pre[t, g] += sum_{valid (f, n) of g} act(z[t, f, n]) / counts[g]
 *           (accumulated: zero `pre` first), z = b[f, n] + sum_k w[f, n, k] x[t, idx(f, k)].
 * Backward: with c1t[g, t] = dL/dpre[t, g] / counts[g] (the reference's c1T) and
 *           dz = c1t * act'(z) on valid slots: dx[t, idx(f, k)] += sum_n dz w[f, n, k],
 *           dw[f, n, k] += sum_t dz x[t, idx(f, k)], db[f, n] += sum_t dz (all accumulated).
 * Activations: GL_ACT_RELU (the layer's Mean(ReLU)) or GL_ACT_IDENTITY. */
typedef struct GlK16Args {
  const float* x;           /* [B, ldx] */
  const uint8_t* env;       /* [G*NB16, 16], 16-byte aligned */
  const int16_t* feat;      /* [Q, S] */
  const int32_t* buckets;   /* [nb, 4], 16-byte aligned */
  const int32_t* q_off;     /* [Q+1] */
  const int32_t* rec_off;   /* [nb+1] */
  const float* w;           /* 16-byte aligned */
  const float* b;           /* 16-byte aligned */
  const int32_t* counts;    /* [G] */
  float* pre;               /* forward: [B, ldp], accumulated */
  const float* c1t;         /* backward: [G, ldc] */
  float* dx;                /* backward: [B, lddx], accumulated */
  float* dw;                /* backward: weight-shaped, accumulated */
  float* db;                /* backward: bias-shaped, accumulated, 16-byte aligned */
  int64_t B, D, G, NB16, Q, S;
  int64_t nbuckets;         /* rows of `buckets` (q_off values are clamped to it) */
  int64_t ldx, ldp, ldc, lddx;
  int32_t act;              /* GL_ACT_RELU or GL_ACT_IDENTITY */
  int32_t tokens;           /* token chunk per block (0 = automatic; else a multiple of 64 for the
                               forward, of 32 for the backward, at most 1024) */
} GlK16Args;

int gl_k16_fwd_f32(const GlK16Args* args, void* stream);
int gl_k16_bwd_f32(const GlK16Args* args, void* stream);
/* Token chunk the automatic choice would use (backward != 0: the backward's), or a negative status. */
int gl_k16_auto_tokens(int64_t B, int64_t S, int32_t backward);
/* The same layer with bf16 parameters (w, b point to bf16 [G*NB16, 16, 16] / [G*NB16, 16]) on the tensor
 * cores, the reference's kgen arithmetic (experimental/kgen/kgen.cuh): x rounded to bf16 as it is staged,
 * every bf16 x bf16 product exact in fp32, the backward's dz carried as hi + lo bf16 ("split" precision).
 * Same arguments, layouts and accumulation as gl_k16_fwd_f32 / gl_k16_bwd_f32 (dw, db fp32); `tokens` =
 * 0 (automatic), 32, 64 or 128 tokens per block; S <= 256. */
int gl_k16_fwd_tc(const GlK16Args* args, void* stream);
/* With `wabsmax` ([G] max |w| over each output's records) and `rowmax` ([nbuckets] per row of `buckets`, the
 * bucket's largest number of record inputs on one local position) the dX tile is int32 fixed point at one
 * power-of-two scale per token and set (16 max|act'| sum_b rowmax_b |c1t[g_b, t]| wabsmax_{g_b} scale <=
 * 2^30; a token whose bound is not finite gets NaN); with both NULL it is fp32. */
int gl_k16_bwd_tc(const GlK16Args* args, const float* wabsmax, const int32_t* rowmax, void* stream);
/* The layer with fp32 parameters (w, b fp32, as gl_k16_fwd_f32 / gl_k16_bwd_f32) on the tensor cores: x, w and
 * dz are each split into three bf16 terms (v = v1 + v2 + v3, exact for 2^-110 <= |v| below bf16's largest value)
 * and every product sum is the six MMAs of the term pairs i + j <= 2, so the results agree with the fp32 SIMT
 * kernels to fp32 rounding (the dropped pairs are below 2^-23 of each |a||b|).  Arguments, `tokens`, S and
 * the optional fixed-point dX bounds as gl_k16_fwd_tc / gl_k16_bwd_tc.  An infinite x, w or dz gives NaN (its
 * second term is inf - inf), where the SIMT kernels may give an infinity. */
int gl_k16_fwd_tc_f32(const GlK16Args* args, void* stream);
int gl_k16_bwd_tc_f32(const GlK16Args* args, const float* wabsmax, const int32_t* rowmax, void* stream);

/* The same forward on the 5th-generation tensor cores (tcgen05 MMAs into TMEM accumulators; no counterpart
 * in the reference, whose kgen kernels use mma.sync): bf16 parameters (gl_k16_fwd_t5, the reference's
 * arithmetic as gl_k16_fwd_tc) or fp32 ones (gl_k16_fwd_t5_f32, three-term bf16 splits as
 * gl_k16_fwd_tc_f32).  Each record's weights are expanded over its set's S positions, so S must be 64
 * (GL_ERR_UNSUPPORTED otherwise) and a record's 16 positions must be distinct (the reference's lowering
 * guarantees both); 128 tokens per block (`tokens` 0 or 128).  `status` (optional, device int32) is set
 * to 1 if a wait for the tensor cores exceeded its iteration limit (the results are then incomplete). */
int gl_k16_fwd_t5(const GlK16Args* args, int32_t* status, void* stream);
int gl_k16_fwd_t5_f32(const GlK16Args* args, int32_t* status, void* stream);
/* The backward on tcgen05 (replaces the reference's kgen K = 16 backward, experimental/kgen/kgen.cuh:202-536;
 * same arguments, layouts and accumulation into dx, dw, db as gl_k16_bwd_tc / gl_k16_bwd_tc_f32, S = 64,
 * distinct positions per record, `tokens` 0 or 128).  dX is summed for each input set in the tensor
 * memory in fp32 (no fixed-point bounds) and added to dx once per set and 128 tokens; dW = dz^T X and
 * db = dz^T 1 are products of the tensor cores as well.  bf16 parameters
 * (gl_k16_bwd_t5): x and w one bf16 term, dz two (hi + lo, the reference's split precision); fp32 ones
 * (gl_k16_bwd_t5_f32): three terms each.  `status` as gl_k16_fwd_t5. */
int gl_k16_bwd_t5(const GlK16Args* args, int32_t* status, void* stream);
int gl_k16_bwd_t5_f32(const GlK16Args* args, int32_t* status, void* stream);

/* Layout of the argument structs, for bindings that declare them field by field (replaces the
 * reference's sp_struct_layout, sparse_pooling/kernels/cuda/abi.cu:25, which its ctypes bridge checks
 * at load, backends/cuda/runtime.py:103-121).  which: 0 GlFwdArgs, 1 GlBwdArgs, 2 GlAdamArgs,
 * 3 GlSharedArgs, 4 GlSetArgs, 5 GlEventArgs, 6 GlK16Args.  gl_struct_layout writes sizeof(struct)
 * and then every field's offset, in declaration order, into out[0 .. n) and returns the number of
 * values (GL_ERR_SHAPE when n is too small, GL_ERR_UNSUPPORTED for an unknown id); gl_struct_fields
 * returns the field names in declaration order, each followed by a comma (NULL for an unknown id). */
#define GL_STRUCT_COUNT 7
int gl_struct_layout(int which, int64_t* out, int n);
const char* gl_struct_fields(int which);

/* Number of kernels this library has launched successfully in this process
   (all devices).  Benchmarks difference it around a timed region. */
int64_t gl_launch_count(void);

/* Token tile the automatic choice would use for input_dim D (forward / backward),
   or a negative status when no tile fits in shared memory. */
int gl_fwd_auto_tokens(int64_t D);
int gl_bwd_auto_tokens(int64_t D);

#ifdef __cplusplus
}
#endif

#endif /* GRANULE_B200_H */
