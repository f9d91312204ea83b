// libnabla_g1: the B200 (sm_100a) batched G1 control step behind the C ABI of include/nabla_g1.h.
//
// k_forward: one warp per world, WPB worlds per block, each world's whole control step (nsub substeps) in one
// launch with its state resident in shared memory (nb_g1_step.cuh), so a step is a single kernel per call.
#include "../../include/nabla_g1.h"
#include <algorithm>
#include <cstddef>
#include <mutex>
#include "nb_g1_step.cuh"
#include "nb_g1_adjoint.cuh"
#include "nb_g1_kin.cuh"
#include "nb_g1_jac.cuh"

namespace nbg1 {

#ifndef NB_WPB
#define NB_WPB 15
#endif
#ifndef NB_LOCKSTEP
#define NB_LOCKSTEP 1
#endif

constexpr int WPB = NB_WPB;  // worlds (warps) per block
// NB_LOCKSTEP: the worlds of a block run their Newton iterations in lockstep (a block barrier per iteration): the
// warps of an SM then fetch the same instructions at the same time, instead of each streaming the ~60 KB Newton loop
// from its own position (the kernel is bound by instruction fetch otherwise). WPB = 10: one block of 10 worlds
// (220 KB of shared memory) per SM, so the whole SM runs one instruction stream (measured: 4.06 ms at B = 4096
// against 4.27 ms with two blocks of 5). NB_LOCKSTEP = -1 keeps one barrier per substep only (the substep
// transitions in step, each world's Newton iterations on their own): 3.81 ms against 3.84 at the same code, and
// it needs the Newton loop to fit the instruction cache (~40 KB measured for 10 warps on separate paths).
constexpr int TAPE_WORDS = REC_WORDS;
constexpr long long ABI_VERSION = 4;  // 2: the tape's L_Q in tree-block order; 3: only its pattern's entries; 4: L_Q
                                      // at the record's end (the compact record: the first REC_COMPACT words)

__global__ void __launch_bounds__(WPB * 32) k_forward(int nw, const float* __restrict__ qpos,
                                                      const float* __restrict__ qvel, const float* __restrict__ warm,
                                                      const float* __restrict__ ctrl, const float* __restrict__ fric,
                                                      const float* __restrict__ com, int iterations, int nsub,
                                                      float* __restrict__ oq, float* __restrict__ ov,
                                                      float* __restrict__ ow, int* __restrict__ info,
                                                      float* __restrict__ ocon, int* __restrict__ stats,
                                                      float* __restrict__ tape, const int* __restrict__ order,
                                                      int tape_words) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = blockIdx.x * (int)(blockDim.x >> 5) + warp;  // the warp's place in the world order (k_order),
                                                                   // or its world index
#if !NB_LOCKSTEP
  if (slot >= nw) return;  // whole warps leave; the block has no block-wide barrier
#endif
  const bool active = slot < nw;  // (lockstep: inactive warps stay for the barriers)
  const int w = active ? (order ? __ldg(order + slot) : slot) : 0;
  World& s = reinterpret_cast<World*>(smem)[warp];
  const size_t w64 = (size_t)(active ? w : 0);
  for (int i = lane; i < NQ; i += 32) s.qpos[i] = qpos[w64 * NQ + i];
  for (int i = lane; i < NV; i += 32) { s.qvel[i] = qvel[w64 * NV + i]; s.qacc[i] = warm[w64 * NV + i]; }
  for (int i = lane; i < NU; i += 32) s.ctrl[i] = ctrl[w64 * NU + i];
  if (lane < 3) s.com[lane] = com[w64 * 3 + lane];
  if (lane == 0) { s.fric = fric[w64]; s.unsup = 0; s.nit = 0; }  // (w64: world 0 for an inactive warp)
  __syncwarp();
  for (int k = 0; k < nsub; k++) {
    float* rec = tape && active ? tape + (w64 * nsub + k) * tape_words : nullptr;
    if (active) substep_pre(s, lane, rec);
#if NB_LOCKSTEP < 0
    // each world iterates on its own; the block meets once, after every world's last iteration
    while (!uall(!active || s.ndone || s.nit_cur >= iterations)) newton_iter(s, lane);
    __syncthreads();
#elif NB_LOCKSTEP
    // rounds of up to NB_LOCKSTEP iterations per world, a block barrier after each round
    while (true) {
      for (int q = 0; q < NB_LOCKSTEP; q++) {
        if (uall(!active || s.ndone || s.nit_cur >= iterations)) break;
        newton_iter(s, lane);
      }
      if (__syncthreads_and(!active || s.ndone || s.nit_cur >= iterations)) break;
    }
#else
    while (!uall(!active || s.ndone || s.nit_cur >= iterations)) newton_iter(s, lane);
#endif
    if (active) substep_post(s, lane, stats ? stats + (w64 * nsub + k) * 8 : nullptr, rec, tape_words == REC_WORDS);
  }
  if (!active) return;
  for (int i = lane; i < NQ; i += 32) oq[w64 * NQ + i] = s.qpos[i];
  for (int i = lane; i < NV; i += 32) { ov[w64 * NV + i] = s.qvel[i]; ow[w64 * NV + i] = s.qacc[i]; }
  if (lane == 0) {
    info[w64 * 4] = s.nit;
    info[w64 * 4 + 1] = s.ncon_raw;
    info[w64 * 4 + 2] = s.nefc;
    info[w64 * 4 + 3] = s.unsup;
  }
  if (ocon)
    for (int c = lane; c < MAXCON; c += 32) {
      float* o = ocon + (w64 * MAXCON + c) * 8;
      const bool v = c < s.ncon;
      o[0] = v ? (float)s.con_pair[c] : -1.f;
      o[1] = v ? s.con_dist[c] : 0.f;
      for (int k = 0; k < 3; k++) {  // (con_pos is kept relative to the root origin O)
        o[2 + k] = v ? s.con_pos[c][k] + s.O[k] : 0.f;
        o[5 + k] = v ? s.con_fr[c][k] : 0.f;
      }
    }
}

constexpr size_t SMEM = sizeof(World) * WPB;

// ---- the world order ----------------------------------------------------------------------------------------------
// A block's ten worlds iterate in lockstep, so the block takes as long as its slowest world, and which worlds share a
// block decides how long the others wait. k_order sorts the worlds by the root height of their input state, lowest
// first, into the order k_forward's blocks take them: a lower root puts more geoms on the floor (more contacts and
// constraint rows, more Newton iterations: the step's iteration count correlates -0.71 with the root height on
// seeded standing states), so a block gets worlds of similar cost and the costliest blocks start first. The
// reference orders its Newton kernel's worlds by constraint-row count for the same reason (g1_engine/host.py:
// 229-298, from its split forward's first kernel); the fused step has no such pre-pass, so the key is an input.
// The key orders the worlds of each chunk of ORD_CHUNK (root height as an ordered unsigned, then the world index:
// distinct keys, so the order is deterministic), and a world's place in its chunk is its rank there, the number of
// the chunk's keys below its own: ORD_TPW threads count it over slices of the chunk's keys, which every block of the
// chunk stages in shared memory, so the sort spreads over ORD_CHUNK / ORD_WPB blocks with one barrier (a bitonic
// sort of the chunk in one block took 40 us at B = 4096, 1.3 % of the step). The outputs do not depend on the
// order (a world's arithmetic is the same in any warp of any block).
constexpr int ORD_CHUNK = 4096, ORD_TPW = 8, ORD_THREADS = 256, ORD_WPB = ORD_THREADS / ORD_TPW;
constexpr int ORD_BLOCKS_PER_CHUNK = ORD_CHUNK / ORD_WPB;
__device__ __forceinline__ unsigned long long order_key(const float* qpos, int w) {
  unsigned u = __float_as_uint(__ldg(qpos + (size_t)w * NQ + 2));
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // the float order as the unsigned order
  return ((unsigned long long)u << 32) | (unsigned)w;
}
__global__ void __launch_bounds__(ORD_THREADS) k_order(int nw, const float* __restrict__ qpos,
                                                       int* __restrict__ order) {
  __shared__ unsigned long long key[ORD_CHUNK];
  const int base = (blockIdx.x / ORD_BLOCKS_PER_CHUNK) * ORD_CHUNK, n = min(ORD_CHUNK, nw - base);
  const int first = (blockIdx.x % ORD_BLOCKS_PER_CHUNK) * ORD_WPB;  // this block's worlds: chunk positions first..
  if (first >= n) return;  // (the whole block)
  for (int i = threadIdx.x; i < n; i += ORD_THREADS) key[i] = order_key(qpos, base + i);
  __syncthreads();
  const int sub = threadIdx.x % ORD_TPW, i = first + threadIdx.x / ORD_TPW;  // i: this group's world
  const unsigned long long mine = i < n ? key[i] : 0ull;
  int rank = 0;
#pragma unroll 4
  for (int v = sub; v < n; v += ORD_TPW) rank += key[v] < mine;
#pragma unroll
  for (int o = ORD_TPW / 2; o > 0; o >>= 1) rank += __shfl_xor_sync(FULL, rank, o);  // the group's lanes
  if (sub == 0 && i < n) order[base + rank] = base + i;
}

// ---- the adjoint ------------------------------------------------------------------------------------------------
// Worlds per block of k_adjoint: up to AWPB (14 x 16.2 KB, one block per SM). The worlds meet at a block barrier
// before every substep, so the SM's warps run the same code together (one instruction stream; measured at B = 4096:
// 1.06 ms against 1.14 ms with one world per block and no barrier). The launch spreads the worlds evenly over whole
// waves: as many waves as AWPB per SM needs, and per block the fewest worlds that fill them (a block's time grows
// with its worlds, but less than in proportion: at B = 4096 on configuration 3, 3 waves of 10 worlds ran in 0.588
// ms, 2.1 waves of 13 in 0.681 ms, 2 waves of 14 in 0.479 ms). Two instances: blocks of up to AWPB_SMALL worlds run
// the one compiled for that many (more registers per thread: 0.588 against 0.605 ms for the same 10-world blocks in
// the 13-world instance), larger blocks the AWPB one.
#ifndef NB_AWPB
#define NB_AWPB 14
#endif
constexpr int AWPB = NB_AWPB, AWPB_SMALL = 10;
struct AdjBlock { AWorld s; Adj a; };
static_assert(offsetof(AdjBlock, a) % 16 == 0 && sizeof(AdjBlock) % 16 == 0, "each world's Adj 16-byte aligned");
constexpr size_t ASMEM = sizeof(AdjBlock) * AWPB;
static_assert(ASMEM <= 227 * 1024 && ASMEM + 1024 <= 228 * 1024, "one adjoint block of AWPB worlds per SM");

// The starting cotangent of one adjoint over nsub records tw (the world's first record): the output cotangent is
// (gq, gv) (qpos form, in any memory), or the unit vector of output row `unit` (0..70: qpos' in qpos form, then qvel')
// when unit >= 0; into A.qout (dof tangent), A.vb, with A.ub cleared
template <class RW>
__device__ __noinline__ void adj_row_init(RW& A, const float* tw, int nsub, int rec_words, const float* gq,
                                          const float* gv, int unit, int normal, int lane) {
  const float h = G1_TIMESTEP;
  if (lane == 0) A.normal = normal;
  auto cq = [&](int i) { return unit >= 0 ? (i == unit ? 1.f : 0.f) : gq[i]; };
  auto cv = [&](int i) { return unit >= 0 ? (i + NQ == unit ? 1.f : 0.f) : gv[i]; };
  for (int i = lane; i < NU; i += 32) A.ub[i] = 0.f;
  for (int i = lane; i < NV; i += 32) A.vb[i] = cv(i);
  // the output cotangent in the dof tangent: the quaternion part at the output quaternion q' (re-integrated from the
  // last record): 1/2 Im(q'* gq) / |q'|^2
  const float* last = tw + (size_t)(nsub - 1) * rec_words;
  for (int i = lane; i < NV; i += 32)
    if (i < 3 || i >= 6) A.qout[i] = cq(i < 3 ? i : i + 1);
  if (lane == 0) {
    float q[4] = {last[T_QPOS + 3], last[T_QPOS + 4], last[T_QPOS + 5], last[T_QPOS + 6]};
    const float wv[3] = {last[T_QVEL + 3] + h * last[T_AADV + 3], last[T_QVEL + 4] + h * last[T_AADV + 4],
                         last[T_QVEL + 5] + h * last[T_AADV + 5]};
    const float nw = sqrtf(dot3(wv, wv));
    if (nw > 0.f) {
      float sa, ca;
      sincosf(0.5f * h * nw, &sa, &ca);
      const float dq[4] = {ca, sa * wv[0] / nw, sa * wv[1] / nw, sa * wv[2] / nw};
      float o[4];
      qmul(q, dq, o);
      const float on = sqrtf(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      for (int k = 0; k < 4; k++) q[k] = o[k] / on;
    }
    const float g[4] = {cq(3), cq(4), cq(5), cq(6)};
    const float qc[4] = {q[0], -q[1], -q[2], -q[3]};
    float m[4];
    qmul(qc, g, m);
    const float n2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    for (int k = 0; k < 3; k++) A.qout[3 + k] = 0.5f * m[1 + k] / n2;
  }
  __syncwarp();
}

// One world's adjoint (one warp): leaves the input cotangents in A.qout (dof tangent), A.vb, A.ub; returns the replay
// flags. block_sync: a block barrier before every substep (every warp of the block calls this with the same nsub).
__device__ __noinline__ int adj_world(AWorld& s, Adj& A, const float* tw, int nsub, int rec_words, float fric,
                                      const float* comw,
                                      const float* ctrlw, const float* gq, const float* gv, int clamp_kv,
                                      float clamp_soft, int normal, int lane, bool block_sync) {
  if (lane == 0) s.fric = fric;
  if (lane < 3) s.com[lane] = comw[lane];
  for (int i = lane; i < NU; i += 32) A.u[i] = ctrlw ? ctrlw[i] : 0.f;
  adj_row_init(A, tw, nsub, rec_words, gq, gv, -1, normal, lane);
  int flags = 0;
  for (int k = nsub - 1; k >= 0; k--) {
    if (block_sync) __syncthreads();  // (the same value on every thread of the block)
    flags |= adj_substep(s, A, tw + (size_t)k * rec_words, rec_words == REC_WORDS, clamp_kv, clamp_soft, A.cw, lane,
                         block_sync);
  }
  return flags;
}

// tape: nw * nsub records; gq_out (B,36) / gv_out (B,35): cotangents of qpos' / qvel'; outputs gq_in (B,36) (qpos
// form), gv_in (B,35), gctrl (B,29), info (B,) (replay mismatch bits); ctrl: the step's setpoints (clamp_kv 2 only)
template <int MAXW>  // the most worlds a block of this instance takes (its register budget follows)
__global__ void __launch_bounds__(MAXW * 32) k_adjoint(int nw, int nsub, const float* __restrict__ tape,
                                                       const float* __restrict__ fric, const float* __restrict__ com,
                                                       const float* __restrict__ gq_out,
                                                       const float* __restrict__ gv_out, float* __restrict__ gq_in,
                                                       float* __restrict__ gv_in, float* __restrict__ gctrl,
                                                       int* __restrict__ info, const float* __restrict__ ctrl,
                                                       float clamp_soft, int clamp_kv, int normal, int tape_words) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int w = blockIdx.x * (int)(blockDim.x >> 5) + warp;  // (blockDim.x / 32 <= AWPB worlds per block)
  const bool active = w < nw;  // inactive warps replay world 0 for the barriers and write nothing
  if (!active) w = 0;
  AdjBlock& blk = reinterpret_cast<AdjBlock*>(smem)[warp];
  AWorld& s = blk.s;
  Adj& A = blk.a;
  const size_t w64 = (size_t)w;
  const float* tw = tape + w64 * nsub * tape_words;
  const int flags = adj_world(s, A, tw, nsub, tape_words, fric[w], com + w64 * 3, ctrl ? ctrl + w64 * NU : nullptr,
                              gq_out + w64 * NQ, gv_out + w64 * NV, clamp_kv, clamp_soft, normal, lane, true);
  if (!active) return;
  // the input qpos gradient in qpos form: (q_lin, 2 xi (0, q_rot), q_hinge), xi the input quaternion
  for (int i = lane; i < NV; i += 32) {
    if (i < 3) gq_in[w64 * NQ + i] = A.qout[i];
    else if (i >= 6) gq_in[w64 * NQ + i + 1] = A.qout[i];
    gv_in[w64 * NV + i] = A.vb[i];
  }
  for (int i = lane; i < NU; i += 32) gctrl[w64 * NU + i] = A.ub[i];
  if (lane == 0) {
    const float xi[4] = {tw[T_QPOS + 3], tw[T_QPOS + 4], tw[T_QPOS + 5], tw[T_QPOS + 6]};
    const float t[4] = {0.f, A.qout[3], A.qout[4], A.qout[5]};
    float o[4];
    qmul(xi, t, o);
    for (int k = 0; k < 4; k++) gq_in[w64 * NQ + 3 + k] = 2.f * o[k];
    info[w] = flags;
  }
}

// The step Jacobian (B, 71, 99): row r = the VJP of output r (qpos' in qpos form 0..35, qvel' 36..70) in the
// tangent columns (qpos tangent 35 | qvel 35 | ctrl 29). One block per world, one lane per right-hand side (the 70
// tangent-basis cotangents of the output; nb_g1_jac.cuh), the record's shared terms prepared once per record by the
// block. info (B,): the replay flags (zeroed by the launcher).
constexpr int JROWS = NQ + NV, JCOLS = 2 * NV + NU;
constexpr size_t JSMEM = sizeof(JBlock);
static_assert(2 * (JSMEM + 1024) <= 228 * 1024, "two Jacobian blocks per SM");
__global__ void __launch_bounds__(JTHREADS, 2) k_jacobian(int nw, int nsub, const float* __restrict__ tape,
                                                          const float* __restrict__ fric,
                                                          const float* __restrict__ com, float* __restrict__ jac,
                                                          int* __restrict__ info, const float* __restrict__ ctrl,
                                                          float clamp_soft, int clamp_kv, int normal, int tape_words) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float qcoef[12];  // the quaternion rows: row 3 + c = sum_k qcoef[3 c + k] (rotation cotangent k)
  JBlock& B = *reinterpret_cast<JBlock*>(smem);
  const int t = threadIdx.x, w = blockIdx.x;
  const size_t w64 = (size_t)w;
  const float* tw = tape + w64 * nsub * tape_words;
  const int j = t < JNR ? t : JNR + (t & 1);  // the lane's right-hand side (spare lanes: the spare columns)
  float* x = B.rhs + j;
  for (int e = t; e < NTRIP; e += JTHREADS) B.R.LQ[e] = 0.f;  // L_Q's entries off its pattern
  if (t == 0) B.R.flags = 0;
  for (int i = 0; i < NV; i++) {
    JX(JO_Q, i) = j < NV && i == j ? 1.f : 0.f;
    JX(JO_V, i) = j >= NV && j < JNR && i == j - NV ? 1.f : 0.f;
  }
  for (int i = 0; i < NU; i++) JX(JO_U, i) = 0.f;
  if (t == 0) {  // the output cotangent of a qpos' quaternion entry in the rotation tangent: 1/2 Im(q'* e_c) / |q'|^2
    const float* last = tw + (size_t)(nsub - 1) * tape_words;
    const float h = G1_TIMESTEP;
    float q[4] = {last[T_QPOS + 3], last[T_QPOS + 4], last[T_QPOS + 5], last[T_QPOS + 6]};
    const float wv[3] = {last[T_QVEL + 3] + h * last[T_AADV + 3], last[T_QVEL + 4] + h * last[T_AADV + 4],
                         last[T_QVEL + 5] + h * last[T_AADV + 5]};
    const float nwv = sqrtf(dot3(wv, wv));
    if (nwv > 0.f) {
      float sa, ca;
      sincosf(0.5f * h * nwv, &sa, &ca);
      const float dq[4] = {ca, sa * wv[0] / nwv, sa * wv[1] / nwv, sa * wv[2] / nwv};
      float o[4];
      qmul(q, dq, o);
      const float on = sqrtf(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      for (int k = 0; k < 4; k++) q[k] = o[k] / on;
    }
    const float qc[4] = {q[0], -q[1], -q[2], -q[3]};
    const float n2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    for (int c = 0; c < 4; c++) {
      const float g[4] = {c == 0 ? 1.f : 0.f, c == 1 ? 1.f : 0.f, c == 2 ? 1.f : 0.f, c == 3 ? 1.f : 0.f};
      float m[4];
      qmul(qc, g, m);
      for (int k = 0; k < 3; k++) qcoef[3 * c + k] = 0.5f * m[1 + k] / n2;
    }
  }
  for (int k = nsub - 1; k >= 0; k--) {
    __syncthreads();  // (the previous record's cotangents are done with the shared terms and lambda / y)
    jac_prep(B, tw + (size_t)k * tape_words, tape_words == REC_WORDS, fric + w, com + 3 * w64,
             ctrl ? ctrl + w64 * NU : nullptr, clamp_soft, clamp_kv, normal, t);
    jac_rhs_solves(B.R, x);
    jac_rhs_sweep(B.R, x);
  }
  __syncthreads();
  float* out = jac + w64 * JROWS * JCOLS;
  for (int e = t; e < JROWS * JCOLS; e += JTHREADS) {
    const int r = e / JCOLS, c = e - r * JCOLS;
    const float* row = B.rhs + (c < NV ? JO_Q + c : (c < 2 * NV ? JO_V + c - NV : JO_U + c - 2 * NV)) * JS;
    float v;
    if (r < 3) v = row[r];
    else if (r < 7) v = qcoef[3 * (r - 3)] * row[3] + qcoef[3 * (r - 3) + 1] * row[4] + qcoef[3 * (r - 3) + 2] * row[5];
    else if (r < NQ) v = row[r - 1];
    else v = row[NV + r - NQ];
    out[e] = v;
  }
  if (t == 0 && B.R.flags) atomicOr(info + w, B.R.flags);
}
// ---- diagnostics: device counters (uint64, DIAG order of the Python layer) added by one small kernel per call ------
enum : int {
  D_FWD_CALLS, D_FWD_WORLDS, D_FWD_UNSUPPORTED, D_FWD_ITER_LIMIT, D_TAPE_RECORDS, D_REFACT_RECORDS, D_NONCONV_RECORDS,
  D_SINGULAR_RECORDS, D_BWD_CALLS, D_BWD_ROWS, D_NONFINITE_ROWS, D_NONFINITE_QPOS, D_NONFINITE_QVEL, D_NONFINITE_CTRL,
  D_NONFINITE_COT, D_REPLAY_MISMATCH, D_FWD_CONTACT_OVERFLOW, D_FWD_ROW_OVERFLOW, NDIAG
};
enum : int { NONFINITE_QPOS = 1, NONFINITE_QVEL = 2, NONFINITE_CTRL = 4, NONFINITE_COT = 8, NONFINITE_SHIFT = 16 };

// a warp's count into counter k (exact integer sums: the totals do not depend on the order)
__device__ __forceinline__ void diag_add(unsigned long long* d, int k, unsigned v) {
  v = __reduce_add_sync(FULL, v);
  if ((threadIdx.x & 31) == 0 && v) atomicAdd(&d[k], (unsigned long long)v);
}
__device__ __forceinline__ bool finite_row(const float* x, int n) {
  bool ok = true;
  for (int i = 0; i < n; i++) ok &= isfinite(x[i]);
  return ok;
}

__global__ void k_diag_fwd(unsigned long long* d, int nw, int nsub, int iterations, const int* info,
                           const float* tape, int tape_words) {
  unsigned unsup = 0, lim = 0, oc = 0, orow = 0, refact = 0, nonconv = 0, sing = 0;
  const int stride = gridDim.x * blockDim.x;
  for (int w0 = blockIdx.x * blockDim.x; w0 < nw; w0 += stride) {  // whole warps stay in the loop
    const int w = w0 + threadIdx.x;
    if (w < nw) {
      const int bits = info[4 * w + 3];
      unsup += bits != 0;
      oc += (bits & CONTACT_OVERFLOW) != 0;
      orow += (bits & ROW_OVERFLOW) != 0;
      lim += info[4 * w] >= iterations;
      if (tape)
        for (int k = 0; k < nsub; k++) {
          const unsigned f = __float_as_uint(tape[((size_t)w * nsub + k) * tape_words + T_FLAGS]);
          refact += (f & TAPE_REFACT) != 0;
          nonconv += (f & TAPE_NONCONV) != 0;
          sing += (f & TAPE_SINGULAR) != 0;
        }
    }
  }
  diag_add(d, D_FWD_UNSUPPORTED, unsup);
  diag_add(d, D_FWD_ITER_LIMIT, lim);
  diag_add(d, D_FWD_CONTACT_OVERFLOW, oc);
  diag_add(d, D_FWD_ROW_OVERFLOW, orow);
  diag_add(d, D_REFACT_RECORDS, refact);
  diag_add(d, D_NONCONV_RECORDS, nonconv);
  diag_add(d, D_SINGULAR_RECORDS, sing);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    atomicAdd(&d[D_FWD_CALLS], 1ull);
    atomicAdd(&d[D_FWD_WORLDS], (unsigned long long)nw);
    if (tape) atomicAdd(&d[D_TAPE_RECORDS], (unsigned long long)nw * nsub);
  }
}

// the backward's counters; the non-finite bits go into info (bits NONFINITE_* << NONFINITE_SHIFT)
__global__ void k_diag_bwd(unsigned long long* d, int nw, const float* gq, const float* gv, const float* gu,
                           const float* cq, const float* cv, int* info) {
  unsigned rows = 0, rq = 0, rv = 0, ru = 0, rc = 0, rm = 0;
  const int stride = gridDim.x * blockDim.x;
  for (int w0 = blockIdx.x * blockDim.x; w0 < nw; w0 += stride) {
    const int w = w0 + threadIdx.x;
    if (w < nw) {
      const size_t ww = (size_t)w;
      const unsigned b = (finite_row(gq + ww * NQ, NQ) ? 0u : (unsigned)NONFINITE_QPOS) |
                         (finite_row(gv + ww * NV, NV) ? 0u : (unsigned)NONFINITE_QVEL) |
                         (finite_row(gu + ww * NU, NU) ? 0u : (unsigned)NONFINITE_CTRL) |
                         (finite_row(cq + ww * NQ, NQ) && finite_row(cv + ww * NV, NV) ? 0u : (unsigned)NONFINITE_COT);
      const int f = info[w];
      info[w] = f | (int)(b << NONFINITE_SHIFT);
      rows += (b & 7u) != 0;
      rq += (b & NONFINITE_QPOS) != 0;
      rv += (b & NONFINITE_QVEL) != 0;
      ru += (b & NONFINITE_CTRL) != 0;
      rc += (b & NONFINITE_COT) != 0;
      rm += (f & ADJ_REPLAY_MISMATCH) != 0;
    }
  }
  diag_add(d, D_NONFINITE_ROWS, rows);
  diag_add(d, D_NONFINITE_QPOS, rq);
  diag_add(d, D_NONFINITE_QVEL, rv);
  diag_add(d, D_NONFINITE_CTRL, ru);
  diag_add(d, D_NONFINITE_COT, rc);
  diag_add(d, D_REPLAY_MISMATCH, rm);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    atomicAdd(&d[D_BWD_CALLS], 1ull);
    atomicAdd(&d[D_BWD_ROWS], (unsigned long long)nw);
  }
}
static unsigned diag_grid(int nw) { return (unsigned)std::max(1, std::min(148, (nw + 255) / 256)); }

// The record of one forward call from its info (B,4): [worlds, contacts summed over the worlds, the most contacts and
// the most constraint rows of one world] (info's counts are the last substep's), written whole into rec and, when
// given, rec2. One block: a strided pass per thread, then a warp and a block reduction (exact integer sums).
constexpr int LAST_THREADS = 256;
__global__ void __launch_bounds__(LAST_THREADS) k_last_forward(int nw, const int* __restrict__ info,
                                                               unsigned* __restrict__ rec, unsigned* __restrict__ rec2) {
  __shared__ unsigned part[3][LAST_THREADS / 32];
  unsigned sum = 0, cmax = 0, rmax = 0;  // (the contact sum modulo 2^32, as every word of the record)
  for (int w = threadIdx.x; w < nw; w += LAST_THREADS) {
    const unsigned c = (unsigned)max(info[4 * w + 1], 0), r = (unsigned)max(info[4 * w + 2], 0);
    sum += c;
    cmax = max(cmax, c);
    rmax = max(rmax, r);
  }
  sum = __reduce_add_sync(FULL, sum);
  cmax = __reduce_max_sync(FULL, cmax);
  rmax = __reduce_max_sync(FULL, rmax);
  const int wid = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { part[0][wid] = sum; part[1][wid] = cmax; part[2][wid] = rmax; }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = 0, c = 0, r = 0;
    for (int i = 0; i < LAST_THREADS / 32; i++) { t += part[0][i]; c = max(c, part[1][i]); r = max(r, part[2][i]); }
    const unsigned v[4] = {(unsigned)nw, t, c, r};
    for (int k = 0; k < 4; k++) {
      rec[k] = v[k];
      if (rec2) rec2[k] = v[k];
    }
  }
}

static_assert(sizeof(World) % 16 == 0, "world records stay 16-byte aligned");
static_assert(offsetof(World, M) % 16 == 0 && offsetof(World, L) % 16 == 0, "float4 copies of the triangles");

}  // namespace nbg1

using namespace nbg1;
#ifdef NB_PROFILE
static size_t g_prof_smem = 0;  // profile builds: a larger dynamic shared-memory size per block (lower occupancy)
#endif

// the SM count of each device (nb_g1_upload records it; 148 until then)
// a record size the tape entries take: the full record or the compact one
static bool tape_words_ok(int w) { return w == REC_WORDS || w == REC_COMPACT; }

static int g_sms[64];
static int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || g_sms[dev] <= 0) return 148;
  return g_sms[dev];
}
// k_adjoint's worlds per block for nw worlds: the waves AWPB per SM needs, filled evenly
static int adjoint_worlds_per_block(int nw) {
  const long long sms = device_sms(), waves = (nw + sms * AWPB - 1) / (sms * AWPB);
  const long long wpb = (nw + sms * waves - 1) / (sms * waves);
  return (int)std::max(1ll, std::min<long long>(AWPB, wpb));
}

extern "C" {

void nb_g1_sizes(long long out[8]) {
  const long long v[8] = {NQ, NV, NU, NB, MAXCON, NEFC, TAPE_WORDS, ABI_VERSION};
  for (int i = 0; i < 8; i++) out[i] = v[i];
}

long long nb_g1_tape_words(int compact) { return compact ? REC_COMPACT : REC_WORDS; }

long long nb_g1_work_bytes(int nw) { return nw < 0 ? -1 : ((long long)nw * (long long)sizeof(int) + 15) / 16 * 16; }

// k_jacobian's leaf-to-root pass visits bodies NB - 1 .. 1 and parks at most one hand-over at a time: every parent
// precedes its children, and a body whose parent is not visited next hands over to the parent already parked, if any
static bool jac_tree_ok() {
  int parent[NB];
  if (cudaMemcpyFromSymbol(parent, g1_body_parent, sizeof(parent)) != cudaSuccess) return false;
  int parked = -1;
  for (int b = NB - 1; b >= 1; b--) {
    if (parked == b) parked = -1;
    if (b < 2) continue;
    const int p = parent[b];
    if (p < 1 || p >= b) return false;
    if (p != b - 1) {
      if (parked != -1 && parked != p) return false;
      parked = p;
    }
  }
  return parked == -1;
}

int nb_g1_upload(const float* consts, cudaStream_t stream) {
  (void)consts;
  (void)stream;
  // the model is compiled in; the per-device work is the kernels' shared-memory opt-in (above 48 KB) and the SM count
  int dev = 0, nsm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return (int)e;
  if (dev >= 0 && dev < 64) g_sms[dev] = nsm;
  e = cudaFuncSetAttribute(k_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_adjoint<AWPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ASMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_adjoint<AWPB_SMALL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(AdjBlock) * AWPB_SMALL));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_jacobian, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)JSMEM);
  if (e == cudaSuccess && !jac_tree_ok()) e = cudaErrorInvalidValue;
  return (int)e;
}

int nb_g1_diag_forward_ex(cudaStream_t stream, unsigned long long* counters, int nw, int nsub, int iterations,
                          const int* info, const float* tape, int tape_words) {
  if (nw < 0 || nsub < 1 || nsub > 32 || !tape_words_ok(tape_words)) return (int)cudaErrorInvalidValue;
  if (!counters || (nw > 0 && !info)) return (int)cudaErrorInvalidValue;
  k_diag_fwd<<<diag_grid(nw), 256, 0, stream>>>(counters, nw, nsub, iterations, info, tape, tape_words);
  return (int)cudaGetLastError();
}

int nb_g1_diag_forward(cudaStream_t stream, unsigned long long* counters, int nw, int nsub, int iterations,
                       const int* info, const float* tape) {
  return nb_g1_diag_forward_ex(stream, counters, nw, nsub, iterations, info, tape, REC_WORDS);
}

int nb_g1_diag_backward(cudaStream_t stream, unsigned long long* counters, int nw, const float* gq, const float* gv,
                        const float* gctrl, const float* gq_out, const float* gv_out, int* info) {
  if (nw < 0 || !counters) return (int)cudaErrorInvalidValue;
  if (nw > 0 && (!gq || !gv || !gctrl || !gq_out || !gv_out || !info)) return (int)cudaErrorInvalidValue;
  k_diag_bwd<<<diag_grid(nw), 256, 0, stream>>>(counters, nw, gq, gv, gctrl, gq_out, gv_out, info);
  return (int)cudaGetLastError();
}

long long nb_g1_diag_count(void) { return NDIAG; }

int nb_g1_last_forward(cudaStream_t stream, int nw, const int* info, unsigned* rec, unsigned* rec2) {
  if (nw < 0 || !rec || (nw > 0 && !info)) return (int)cudaErrorInvalidValue;
  k_last_forward<<<1, LAST_THREADS, 0, stream>>>(nw, info, rec, rec2);
  return (int)cudaGetLastError();
}

int nb_g1_launch(int dev, long long out[8]) {
  for (int i = 0; i < 8; i++) out[i] = 0;
  int old = -1, nsm = 0, fb = 0, ab = 0, jb = 0;
  cudaError_t e = cudaGetDevice(&old);
  if (e != cudaSuccess) return (int)e;
  if ((e = cudaSetDevice(dev)) != cudaSuccess) return (int)e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fb, k_forward, WPB * 32, SMEM);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ab, k_adjoint<AWPB>, AWPB * 32, ASMEM);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&jb, k_jacobian, JTHREADS, JSMEM);
  const cudaError_t e2 = cudaSetDevice(old);
  if (e == cudaSuccess) e = e2;
  if (e != cudaSuccess) return (int)e;
  const long long v[8] = {(long long)SMEM, (long long)fb * WPB, (long long)ASMEM, (long long)ab * AWPB,
                          (long long)JSMEM, (long long)jb * JNR, nsm, 0};
  for (int i = 0; i < 8; i++) out[i] = v[i];
  return 0;
}

int nb_g1_kinematics(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* com,
                     float* qpos_n, float* xpos, float* xquat, float* cvel, float* subtree_com) {
  if (nw < 0) return (int)cudaErrorInvalidValue;
  if (nw == 0) return 0;
  if (!qpos || !qvel || !com || !qpos_n || !xpos || !xquat || !cvel || !subtree_com) return (int)cudaErrorInvalidValue;
  k_kin<<<(nw + KWPB - 1) / KWPB, KWPB * 32, 0, stream>>>(nw, qpos, qvel, com, qpos_n, xpos, xquat, cvel, subtree_com);
  return (int)cudaGetLastError();
}

int nb_g1_kinematics_vjp(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* com,
                         const float* g_qpos_n, const float* g_xpos, const float* g_xquat, const float* g_cvel,
                         const float* g_subtree_com, const float* gq_in, const float* gv_in, float* gq, float* gv) {
  if (nw < 0) return (int)cudaErrorInvalidValue;
  if (nw == 0) return 0;
  if (!qpos || !qvel || !com || !g_qpos_n || !g_xpos || !g_xquat || !g_cvel || !g_subtree_com || !gq || !gv)
    return (int)cudaErrorInvalidValue;
  k_kin_vjp<<<(nw + KWPB - 1) / KWPB, KWPB * 32, 0, stream>>>(nw, qpos, qvel, com, g_qpos_n, g_xpos, g_xquat, g_cvel,
                                                              g_subtree_com, gq_in, gv_in, gq, gv);
  return (int)cudaGetLastError();
}

int nb_g1_jacobian_ex(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction,
                      const float* com, float* jac, int* info, const float* ctrl, float clamp_soft, int clamp_kv,
                      int normal, int tape_words) {
  if (nw < 0 || nsub < 1 || nsub > 32 || clamp_kv < 0 || clamp_kv > 2 || normal < 0 || normal > 3 ||
      !tape_words_ok(tape_words))
    return (int)cudaErrorInvalidValue;
  if (nw == 0) return 0;
  if (!tape || !friction || !com || !jac || !info) return (int)cudaErrorInvalidValue;
  if (clamp_kv == 2 && !ctrl) return (int)cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(info, 0, sizeof(int) * (size_t)nw, stream);
  if (e != cudaSuccess) return (int)e;
  k_jacobian<<<(unsigned)nw, JTHREADS, JSMEM, stream>>>(nw, nsub, tape, friction, com, jac, info, ctrl, clamp_soft,
                                                         clamp_kv, normal, tape_words);
  return (int)cudaGetLastError();
}

int nb_g1_jacobian(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction, const float* com,
                   float* jac, int* info, const float* ctrl, float clamp_soft, int clamp_kv, int normal) {
  return nb_g1_jacobian_ex(stream, nw, nsub, tape, friction, com, jac, info, ctrl, clamp_soft, clamp_kv, normal,
                           REC_WORDS);
}

int nb_g1_adjoint_ex(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction,
                     const float* com, const float* gq_out, const float* gv_out, float* gq_in, float* gv_in,
                     float* gctrl, int* info, const float* ctrl, float clamp_soft, int clamp_kv, int normal,
                     int tape_words) {
  if (nw < 0 || nsub < 1 || nsub > 32 || clamp_kv < 0 || clamp_kv > 2 || normal < 0 || normal > 3 ||
      !tape_words_ok(tape_words))
    return (int)cudaErrorInvalidValue;
  if (nw == 0) return 0;
  if (!tape || !friction || !com || !gq_out || !gv_out || !gq_in || !gv_in || !gctrl || !info)
    return (int)cudaErrorInvalidValue;
  if (clamp_kv == 2 && !ctrl) return (int)cudaErrorInvalidValue;
  const int wpb = adjoint_worlds_per_block(nw);
  const int blocks = (nw + wpb - 1) / wpb;
  auto kernel = wpb <= AWPB_SMALL ? k_adjoint<AWPB_SMALL> : k_adjoint<AWPB>;
  kernel<<<blocks, wpb * 32, sizeof(AdjBlock) * wpb, stream>>>(nw, nsub, tape, friction, com, gq_out, gv_out, gq_in,
                                                               gv_in, gctrl, info, ctrl, clamp_soft, clamp_kv,
                                                               normal, tape_words);
  return (int)cudaGetLastError();
}

int nb_g1_adjoint(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction, const float* com,
                  const float* gq_out, const float* gv_out, float* gq_in, float* gv_in, float* gctrl, int* info,
                  const float* ctrl, float clamp_soft, int clamp_kv, int normal) {
  return nb_g1_adjoint_ex(stream, nw, nsub, tape, friction, com, gq_out, gv_out, gq_in, gv_in, gctrl, info, ctrl,
                          clamp_soft, clamp_kv, normal, REC_WORDS);
}

static int launch_forward(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                          const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                          float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape,
                          int* stats, int* order, int tape_words = REC_WORDS) {
  if (nw < 0 || nsub < 1 || nsub > 32 || iterations < 0 || !tape_words_ok(tape_words))
    return (int)cudaErrorInvalidValue;
  if (nw == 0) return 0;
  if (!qpos || !qvel || !warm || !ctrl || !friction || !com || !qpos_out || !qvel_out || !warm_out || !info)
    return (int)cudaErrorInvalidValue;
  // worlds per block: WPB, or when every world fits one wave of WPB per SM, the fewest that put a block on every SM
  // (a block's time is its slowest world's, so smaller blocks on all SMs beat full blocks on a few); from two waves
  // on, full blocks (measured: blocks of 14 spread evenly over two waves ran 1 % slower than 15)
  int wpb = WPB;
#if !defined(NB_PROFILE) && !defined(NB_FWD_NO_SPREAD)
  {
    const int sms = device_sms();
    if (nw <= sms * WPB) wpb = std::max(1, (nw + sms - 1) / sms);
  }
#endif
  const int blocks = (nw + wpb - 1) / wpb;
#ifdef NB_PROFILE
  const size_t smem = g_prof_smem > SMEM ? g_prof_smem : SMEM;
  if (smem != SMEM) cudaFuncSetAttribute(k_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
#else
  const size_t smem = sizeof(World) * wpb;
#endif
  if (order) {
    k_order<<<(nw + ORD_CHUNK - 1) / ORD_CHUNK * ORD_BLOCKS_PER_CHUNK, ORD_THREADS, 0, stream>>>(nw, qpos, order);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
  }
  k_forward<<<blocks, wpb * 32, smem, stream>>>(nw, qpos, qvel, warm, ctrl, friction, com, iterations, nsub, qpos_out,
                                                qvel_out, warm_out, info, ocon, stats, tape, order, tape_words);
  return (int)cudaGetLastError();
}

int nb_g1_forward(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                  const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                  float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape, void* work) {
  return launch_forward(stream, nw, qpos, qvel, warm, ctrl, friction, com, iterations, nsub, qpos_out, qvel_out,
                        warm_out, info, ocon, tape, nullptr, static_cast<int*>(work));
}

int nb_g1_forward_ex(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                     const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                     float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape,
                     void* work, int tape_words) {
  return launch_forward(stream, nw, qpos, qvel, warm, ctrl, friction, com, iterations, nsub, qpos_out, qvel_out,
                        warm_out, info, ocon, tape, nullptr, static_cast<int*>(work), tape_words);
}

int nb_g1_forward_stats(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                        const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                        float* qpos_out, float* qvel_out, float* warm_out, int* info, int* stats) {
  if (!stats) return (int)cudaErrorInvalidValue;
  return launch_forward(stream, nw, qpos, qvel, warm, ctrl, friction, com, iterations, nsub, qpos_out, qvel_out,
                        warm_out, info, nullptr, nullptr, stats, nullptr);
}

}  // extern "C"

// ---- the forward without caller memory (nb_g1_forward_noalloc) ---------------------------------------------------
// For callers that cannot allocate device memory, the world order of nb_g1_forward's work memory lives in this
// library's own buffer: a fixed array in device memory, one copy per device, loaded with the library. Host code must
// not pass the array's name to a kernel (on the host it names a host-side shadow, not device memory): each device's
// address comes from cudaGetSymbolAddress, looked up on the first call made with that device current and kept.
static __device__ __align__(256) int g_noalloc_order[NB_G1_NOALLOC_MAX_WORLDS];
constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mutex;
static int* g_noalloc_addr[NOALLOC_MAX_DEVICES] = {};

static int noalloc_order_address(int** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_order);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_addr[dev] = static_cast<int*>(p);
  }
  *out = g_noalloc_addr[dev];
  return 0;
}

extern "C" {

int nb_g1_forward_noalloc(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                          const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                          float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape) {
  if (nw > NB_G1_NOALLOC_MAX_WORLDS) return (int)cudaErrorInvalidValue;  // the buffer's capacity
  if (nw <= 0) return nw < 0 ? (int)cudaErrorInvalidValue : 0;
  int* order = nullptr;
  const int rc = noalloc_order_address(&order);
  if (rc) return rc;
  return launch_forward(stream, nw, qpos, qvel, warm, ctrl, friction, com, iterations, nsub, qpos_out, qvel_out,
                        warm_out, info, ocon, tape, nullptr, order);
}

#ifdef NB_PROFILE
// profile builds only: read and clear the phase counters (not part of the product ABI)
int nb_g1_profile_set_smem(long long bytes) {
  g_prof_smem = (size_t)bytes;
  return 0;
}
int nb_g1_profile_read(unsigned long long* out, int n) {
  unsigned long long h[NPROF] = {};
  cudaError_t e = cudaMemcpyFromSymbol(h, g_prof, sizeof(h));
  if (e != cudaSuccess) return (int)e;
  for (int i = 0; i < n && i < NPROF; i++) out[i] = h[i];
  unsigned long long z[NPROF] = {};
  return (int)cudaMemcpyToSymbol(g_prof, z, sizeof(z));
}
#endif
}  // extern "C"
