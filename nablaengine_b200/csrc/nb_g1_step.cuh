// Device code of one G1 substep, one warp per world, the world's state in shared memory (struct World).
//
// Algorithm (reference OamIcs/NablaEngine, src/nablaengine/g1_engine/): forward kinematics, Newton-Euler bias forces
// and the joint-space mass matrix (source.py:181-334), PD actuation clamped to the joint force range (step.py:
// 1762-1778), collision of the 502 explicit pairs with MuJoCo Warp's sphere / capsule / plane primitives (step.py:
// 436-556, 1043-1145), hinge-limit and pyramidal contact rows with refsafe impedance (step.py:1881-1957, 1147-1188),
// the primal Newton solver with an exact line search (step.py:1969-2137) and implicitfast integration (step.py:
// 2153-2182). The layout and the parallel decomposition are this library's own:
//  * lanes own bodies (tree sweeps one depth level at a time), dofs (mass-matrix rows, actuation, J' f), pairs
//    (broad phase), candidate pairs (narrow phase), contacts and constraint rows;
//  * every dof's motion vector about the root origin O is kept (dw = angular, dv = velocity of the point O), and a
//    contact keeps its frame rows and their moments (pos - O) x row: a contact row's Jacobian entry is then
//    frame . dv + moment . dw, so no per-contact Jacobian is stored; J v for all contacts comes from the bodies'
//    spatial velocities at O (one pass over each body's ancestor dofs), and J' f from the contacts' wrenches at O;
//  * contacts are numbered deterministically: pair order, then the pair's contact slot (a ballot prefix sum over the
//    candidates), so results are bitwise reproducible run to run.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define NB_REAL float
#define NB_MODEL_CONST static __device__ const
#include "g1_model_data.h"

namespace nbg1 {

constexpr int NQ = G1_NQ, NV = G1_NV, NU = G1_NU, NB = G1_NBODY, NG = G1_NGEOM, NP = G1_NPAIR;
constexpr int MAXCON = 64, NEFC = 192, KDOF = 16, MAXD = G1_MAXDEPTH;  // the capacity of the ABI and the tape
#ifndef NB_WCON
#define NB_WCON 64
#endif
#ifndef NB_WROWS
#define NB_WROWS 192
#endif
constexpr int WCON = NB_WCON, WROWS = NB_WROWS;  // the capacity of a World record (contacts, constraint rows)
static_assert(WCON <= MAXCON && WROWS <= NEFC && WCON % 32 == 0 && WROWS % 32 == 0, "World capacity");
static_assert(G1_NV == G1_NBODY + 4, "dof d >= 6 is the hinge of body d - 4 (one hinge per body after the root)");
__host__ __device__ constexpr int TRI(int i, int j) { return i * (i + 1) / 2 + j; }  // packed lower triangle, j <= i
constexpr int NTRI = NV * (NV + 1) / 2;
constexpr int NTRIP = (NTRI + 3) / 4 * 4;  // the packed triangles' storage in World: whole float4s

constexpr unsigned FULL = 0xffffffffu;
constexpr int ROWS_PER_LANE = (WROWS + 31) / 32;

enum : int { UNSUPPORTED_PAIR = 1, CONTACT_OVERFLOW = 4, ROW_OVERFLOW = 16 };

// The forward tape: one record of REC_WORDS float32 words per world and substep (record w * nsub + k), what the
// adjoint reads: the substep's input state, the Newton solution a*, a_adv = (M + h kv)^-1 M a*, the Cholesky factor
// of the Newton Hessian at the final zones (L_H, dof order) with its inverse diagonal, the contact table (pair | slot
// << 9, two 16-bit entries per word, contact order), the rows' final zone bits, the actuator clamp mask (dof bits), a
// header and flags, then the factor of M + h kv (L_Q, tree-block order: tb_factor, only the entries of its pattern)
// with its inverse diagonal. The compact tape's records are the first REC_COMPACT words of these (no L_Q: its reader
// rebuilds M + h kv from the replayed poses and factors it).
constexpr int T_QPOS = 0, T_QVEL = 36, T_ASTAR = 71, T_AADV = 106, T_DINVH = 141, T_LH = 176;
constexpr int NTB_TAPE = 341;  // the tree-block factor's pattern (NTB, checked below)
constexpr int T_CON = T_LH + NTRI, T_ZONE = T_CON + MAXCON / 2, T_CLAMP = T_ZONE + NEFC / 32;
constexpr int T_HDR = T_CLAMP + 2, T_FLAGS = T_HDR + 1, REC_COMPACT = T_FLAGS + 1;
constexpr int T_DINVQ = REC_COMPACT, T_LQ = T_DINVQ + NV, REC_WORDS = T_LQ + NTB_TAPE;
static_assert(REC_COMPACT == 848 && REC_WORDS == 1224 && REC_COMPACT % 4 == 0 && REC_WORDS % 4 == 0, "tape layout");
// TAPE_SINGULAR: a pivot of the recorded Hessian factor was clamped (at 1e-30: not positive definite in float32)
enum : unsigned { TAPE_REFACT = 1u << 8, TAPE_NONCONV = 1u << 9, TAPE_SINGULAR = 1u << 12 };
enum : unsigned char { ROW_LIMIT = 0, ROW_PYRAMID = 1, ROW_NORMAL = 2 };

// Phase profile (build with -DNB_PROFILE; the product build has none of it): lane 0 of every world adds the clock64
// cycles since the previous mark to g_prof[phase]; counters from phase 16 on count events.
#ifdef NB_PROFILE
constexpr int NPROF = 40;
__device__ unsigned long long g_prof[NPROF];
#define PROF_START(s) do { __syncwarp(); if (lane == 0) (s).prof_t = clock64(); } while (0)
#define PROF(s, k) do { __syncwarp(); if (lane == 0) { long long t_ = clock64(); \
    atomicAdd(&g_prof[k], (unsigned long long)(t_ - (s).prof_t)); (s).prof_t = t_; } __syncwarp(); } while (0)
#define PROF_COUNT(k, n) do { if (lane == 0) atomicAdd(&g_prof[k], (unsigned long long)(n)); } while (0)
#else
#define PROF_START(s) do { } while (0)
#define PROF(s, k) do { } while (0)
#define PROF_COUNT(k, n) do { } while (0)
#endif

// The world record, resident in shared memory for the whole control step. Its scratch overlaps by phase: the smooth
// phase's body terms (sm: kinematics to mass_and_force) share their space with everything from collision on (the
// contacts, their groups and rows), and the collision phase's geom poses and candidate list (col) with the rows,
// which make_rows writes after collision; what a phase reads was written in the same substep after the previous
// owner of that space was done with it.
struct __align__(16) World {
  float M[NTRIP], L[NTRIP];            // mass matrix (with armature), factor scratch (16-byte aligned)
  float qpos[NQ], qvel[NV], qacc[NV], ctrl[NU], com[3], fric;
  float O[3];                          // the root origin (body 1's position): the moments' reference point
  float dw[NV][3], dv[NV][3];          // dof motion about O: angular axis, velocity of the point O
  float qsm[NV], qacc0[NV], Ma[NV], grad[NV], p[NV], dinv[NV + 1];  // p: the Newton direction, then a_adv
  struct { float K[21], P[KDOF][6]; unsigned char dof[KDOF]; } hs;  // Hessian assembly
  int ngroup, nls, nfact, pad3_;        // groups; line-search evaluations, factorisations (work counters)
  float ncost;                          // Newton state between iterations: cost, iterations, converged, same zones
  int nit_cur, ndone, nsame;
  unsigned clamp_lo, clamp_hi;          // actuator force at its limit (dof bits), for the tape
  int ncon, ncon_raw, nefc, nlim, unsup, ncand, nit, pad_;
  unsigned long long lim_mask;          // dofs with a limit row (rows 0 .. nlim - 1 in dof order)
  union {
    struct {  // from kinematics to the geom poses at the start of collision
      float Q[NB][4], X[NB][3];         // body orientations and positions
      struct { float om[NB][3], al[NB][3], ao[NB][3], wr[NB][6], I[NB][10]; } sm;  // smooth phase
    };
    struct {  // collision on
      unsigned char grp_first[WCON + 1];  // the groups' members: grp_mem[grp_first[g] .. grp_first[g + 1]),
      unsigned char grp_mem[WCON];        // in contact order (group g: the contacts between one body pair)
      int con_pair[WCON];
      unsigned char con_slot[WCON], con_row0[WCON], con_nrow[WCON];
      unsigned short con_bb[WCON];        // the contact's bodies b1 | b2 << 8 (contact_setup on)
      float con_dist[WCON], con_mu[WCON];
      float con_fr[WCON][6];              // frame rows: normal, tangent 1 (tangent 2 = normal x tangent 1)
      float con_pos[WCON][3];
      union {  // per-contact scratch, each consumed by the phase that writes it
        float jd[WCON][3];  // J_d v per frame row
        float wr[WCON][6];  // the contact wrench at O (moment, force)
        struct { int key[WCON]; unsigned char lead[WCON], grp[WCON]; } g;  // contact_setup: the groups
      } cs;
      union {
        struct {  // make_rows on
          float efc_D[WROWS];
          float efc_jar[WROWS];           // J a - aref at the current acceleration a (from make_rows to the
                                          // Newton start: aref)
          short efc_a[WROWS];             // dof (limit row) or contact
          signed char efc_b[WROWS];       // limit sign, or the contact row t (n + mu t1, n - mu t1, n + mu t2, ...)
          unsigned char efc_kind[WROWS];
        };
        struct { float gx[NG][3], gq[NG][4]; unsigned short cand[NP + 2]; } col;  // collision phase
      };
    };
  };
#ifdef NB_PROFILE
  long long prof_t;
#endif
};

// collision computes the geom poses from Q and X into col, then writes the contacts (over Q and X): Q and X must not
// share col's space
static_assert(offsetof(World, Q) + sizeof(World::Q) <= offsetof(World, col) &&
              offsetof(World, X) + sizeof(World::X) <= offsetof(World, col), "Q, X and col overlap");

// ---- small vector helpers --------------------------------------------------------------------------------------
__device__ __forceinline__ void qmul(const float* a, const float* b, float* o) {
  float w = a[0] * b[0] - a[1] * b[1] - a[2] * b[2] - a[3] * b[3];
  float x = a[0] * b[1] + a[1] * b[0] + a[2] * b[3] - a[3] * b[2];
  float y = a[0] * b[2] - a[1] * b[3] + a[2] * b[0] + a[3] * b[1];
  float z = a[0] * b[3] + a[1] * b[2] - a[2] * b[1] + a[3] * b[0];
  o[0] = w; o[1] = x; o[2] = y; o[3] = z;
}
__device__ __forceinline__ void cross(const float* a, const float* b, float* o) {
  float x = a[1] * b[2] - a[2] * b[1], y = a[2] * b[0] - a[0] * b[2], z = a[0] * b[1] - a[1] * b[0];
  o[0] = x; o[1] = y; o[2] = z;
}
__device__ __forceinline__ float dot3(const float* a, const float* b) {
  return a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
}
__device__ __forceinline__ void qrot(const float* q, const float* v, float* o) {  // o = q v q^-1
  float t[3], u[3];
  const float qv[3] = {q[1], q[2], q[3]};
  cross(qv, v, t);
  for (int k = 0; k < 3; k++) t[k] *= 2.f;
  cross(qv, t, u);
  for (int k = 0; k < 3; k++) o[k] = v[k] + q[0] * t[k] + u[k];
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
// Values that are the same on every lane of the warp (a count in shared memory, a warp_sum result; the xor butterfly
// gives every lane the same bits) made provably uniform for the compiler, so branches on them need no divergence
// handling around the shuffles they enclose: uni for counts >= 0, uall for conditions
__device__ __forceinline__ int uni(int x) { return (int)__reduce_max_sync(FULL, (unsigned)x); }
__device__ __forceinline__ bool uall(bool c) { return __all_sync(FULL, c); }
__device__ __forceinline__ float ld(const float* p) { return __ldg(p); }
__device__ __forceinline__ int ldi(const int* p) { return __ldg(p); }

// M(i, j) of a symmetric matrix stored as its packed lower triangle
__device__ __forceinline__ float sym(const float* A, int i, int j) { return j <= i ? A[TRI(i, j)] : A[TRI(j, i)]; }

// ---- smooth dynamics ---------------------------------------------------------------------------------------------
// Forward kinematics with velocities and the velocity-product accelerations (qacc = 0; gravity enters as the
// base acceleration -g), one depth level at a time (lane = body).
__device__ __noinline__ void kinematics(World& s, int lane) {
  const int b = lane;
  const int depth = b < NB ? ldi(g1_body_depth + b) : -1;
  if (lane == 0) {
    s.Q[0][0] = 1.f; s.Q[0][1] = s.Q[0][2] = s.Q[0][3] = 0.f;
    for (int k = 0; k < 3; k++) { s.X[0][k] = 0.f; }
  }
  for (int L = 1; L <= MAXD; L++) {
    if (depth == L) {
      if (b == 1) {
        float q[4] = {s.qpos[3], s.qpos[4], s.qpos[5], s.qpos[6]};
        float n = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
        for (int k = 0; k < 4; k++) s.Q[1][k] = q[k] / n;
        float wl[3] = {s.qvel[3], s.qvel[4], s.qvel[5]}, om[3];
        qrot(s.Q[1], wl, om);
        for (int k = 0; k < 3; k++) {
          s.X[1][k] = s.O[k] = s.qpos[k];
          s.sm.om[1][k] = om[k];
          s.sm.al[1][k] = 0.f;
          s.sm.ao[1][k] = 0.f;
        }
        s.sm.ao[1][2] = -G1_GRAVITY_Z;
      } else {
        const int p = ldi(g1_body_parent + b);
        float Qp[4], Xp[3], omp[3], alp[3], aop[3];
        for (int k = 0; k < 4; k++) Qp[k] = s.Q[p][k];
        for (int k = 0; k < 3; k++) {
          Xp[k] = s.X[p][k]; omp[k] = s.sm.om[p][k];
          alp[k] = s.sm.al[p][k]; aop[k] = s.sm.ao[p][k];
        }
        const float bq[4] = {ld(g1_body_quat + 4 * b), ld(g1_body_quat + 4 * b + 1), ld(g1_body_quat + 4 * b + 2),
                             ld(g1_body_quat + 4 * b + 3)};
        const float bp[3] = {ld(g1_body_pos + 3 * b), ld(g1_body_pos + 3 * b + 1), ld(g1_body_pos + 3 * b + 2)};
        const float ax[3] = {ld(g1_body_axis + 3 * b), ld(g1_body_axis + 3 * b + 1), ld(g1_body_axis + 3 * b + 2)};
        const int d = ldi(g1_body_dofadr + b);
        const float ang = s.qpos[d + 1], qd = s.qvel[d];
        float q0[4], sn, cs, t[3], X[3], Q[4];
        qmul(Qp, bq, q0);
        qrot(Qp, bp, t);
        for (int k = 0; k < 3; k++) X[k] = Xp[k] + t[k];
        sincosf(0.5f * ang, &sn, &cs);
        const float ha[4] = {cs, sn * ax[0], sn * ax[1], sn * ax[2]};
        qmul(q0, ha, Q);
        float aw[3], r[3], wd[3], u1[3], u2[3], u3[3];
        qrot(Q, ax, aw);
        for (int k = 0; k < 3; k++) { r[k] = X[k] - Xp[k]; wd[k] = aw[k] * qd; }
        cross(omp, r, u1);
        cross(omp, wd, u2);
        cross(alp, r, u3);
        float wr_[3];
        cross(omp, u1, wr_);
        for (int k = 0; k < 4; k++) s.Q[b][k] = Q[k];
        for (int k = 0; k < 3; k++) {
          s.X[b][k] = X[k];
          s.sm.om[b][k] = omp[k] + wd[k];
          s.sm.al[b][k] = alp[k] + u2[k];
          s.sm.ao[b][k] = aop[k] + u3[k] + wr_[k];
        }
      }
    }
    __syncwarp();
  }
}

// the dofs' motion vectors about O = the root origin (lane = dof)
__device__ __noinline__ void dof_motion(World& s, int lane) {
  const float O[3] = {s.O[0], s.O[1], s.O[2]};
  for (int i = lane; i < NV; i += 32) {
    float w[3] = {0.f, 0.f, 0.f}, v[3] = {0.f, 0.f, 0.f};
    if (i < 3) {
      v[i] = 1.f;
    } else if (i < 6) {
      float e[3] = {0.f, 0.f, 0.f};
      e[i - 3] = 1.f;
      qrot(s.Q[1], e, w);
    } else {
      const int b = ldi(g1_dof_body + i);
      const float ax[3] = {ld(g1_body_axis + 3 * b), ld(g1_body_axis + 3 * b + 1), ld(g1_body_axis + 3 * b + 2)};
      qrot(s.Q[b], ax, w);
      const float r[3] = {O[0] - s.X[b][0], O[1] - s.X[b][1], O[2] - s.X[b][2]};
      cross(w, r, v);
    }
    for (int k = 0; k < 3; k++) { s.dw[i][k] = w[k]; s.dv[i][k] = v[k]; }
  }
  __syncwarp();
}

// per body: the Newton-Euler wrench at O and the spatial inertia about O (lane = body), then both summed over
// subtrees (leaves first)
__device__ __noinline__ void body_terms(World& s, int lane) {
  const int b = lane;
  const float O[3] = {s.O[0], s.O[1], s.O[2]};
  if (b >= 1 && b < NB) {
    float ip[3] = {ld(g1_body_ipos + 3 * b), ld(g1_body_ipos + 3 * b + 1), ld(g1_body_ipos + 3 * b + 2)};
    if (b == G1_TORSO)
      for (int k = 0; k < 3; k++) ip[k] += s.com[k];
    float c[3], Q[4], om[3], al[3], ao[3];
    for (int k = 0; k < 4; k++) Q[k] = s.Q[b][k];
    for (int k = 0; k < 3; k++) { om[k] = s.sm.om[b][k]; al[k] = s.sm.al[b][k]; ao[k] = s.sm.ao[b][k]; }
    qrot(Q, ip, c);
    const float iq[4] = {ld(g1_body_iquat + 4 * b), ld(g1_body_iquat + 4 * b + 1), ld(g1_body_iquat + 4 * b + 2),
                         ld(g1_body_iquat + 4 * b + 3)};
    float qi[4], R[3][3];
    qmul(Q, iq, qi);
    for (int k = 0; k < 3; k++) {
      float e[3] = {0.f, 0.f, 0.f}, col[3];
      e[k] = 1.f;
      qrot(qi, e, col);
      for (int r = 0; r < 3; r++) R[r][k] = col[r];
    }
    const float In[3] = {ld(g1_body_inertia + 3 * b), ld(g1_body_inertia + 3 * b + 1), ld(g1_body_inertia + 3 * b + 2)};
    float I[3][3];
    for (int r = 0; r < 3; r++)
      for (int q = r; q < 3; q++) {
        float v = R[r][0] * In[0] * R[q][0] + R[r][1] * In[1] * R[q][1] + R[r][2] * In[2] * R[q][2];
        I[r][q] = v; I[q][r] = v;
      }
    const float m = ld(g1_body_mass + b);
    // COM acceleration (qacc = 0) and the inertial wrench about the COM
    float u1[3], u2[3], u3[3], ac[3], F[3], Iom[3], Ial[3], N[3];
    cross(al, c, u1);
    cross(om, c, u2);
    cross(om, u2, u3);
    for (int k = 0; k < 3; k++) { ac[k] = ao[k] + u1[k] + u3[k]; F[k] = m * ac[k]; }
    for (int r = 0; r < 3; r++) {
      Iom[r] = I[r][0] * om[0] + I[r][1] * om[1] + I[r][2] * om[2];
      Ial[r] = I[r][0] * al[0] + I[r][1] * al[1] + I[r][2] * al[2];
    }
    cross(om, Iom, u1);
    // moment arm from O to the COM
    float cO[3], mo[3];
    for (int k = 0; k < 3; k++) cO[k] = s.X[b][k] + c[k] - O[k];
    cross(cO, F, mo);
    for (int k = 0; k < 3; k++) { N[k] = Ial[k] + u1[k] + mo[k]; }
    for (int k = 0; k < 3; k++) { s.sm.wr[b][k] = N[k]; s.sm.wr[b][3 + k] = F[k]; }
    // spatial inertia about O: rotational inertia about O (xx yy zz xy xz yz), h = m cO, m
    const float cc = dot3(cO, cO);
    float* J = s.sm.I[b];
    J[0] = I[0][0] + m * (cc - cO[0] * cO[0]);
    J[1] = I[1][1] + m * (cc - cO[1] * cO[1]);
    J[2] = I[2][2] + m * (cc - cO[2] * cO[2]);
    J[3] = I[0][1] - m * cO[0] * cO[1];
    J[4] = I[0][2] - m * cO[0] * cO[2];
    J[5] = I[1][2] - m * cO[1] * cO[2];
    J[6] = m * cO[0]; J[7] = m * cO[1]; J[8] = m * cO[2]; J[9] = m;
  }
  __syncwarp();
  const int depth = b < NB ? ldi(g1_body_depth + b) : -1;
  const int nch = b < NB ? ldi(g1_body_nchild + b) : 0;
  for (int L = MAXD - 1; L >= 1; L--) {
    if (depth == L && nch > 0) {
      float wr[6], I[10];
      for (int k = 0; k < 6; k++) wr[k] = s.sm.wr[b][k];
      for (int k = 0; k < 10; k++) I[k] = s.sm.I[b][k];
      for (int c = 0; c < nch; c++) {
        const int ch = ldi(g1_body_child + 3 * b + c);
        for (int k = 0; k < 6; k++) wr[k] += s.sm.wr[ch][k];
        for (int k = 0; k < 10; k++) I[k] += s.sm.I[ch][k];
      }
      for (int k = 0; k < 6; k++) s.sm.wr[b][k] = wr[k];
      for (int k = 0; k < 10; k++) s.sm.I[b][k] = I[k];
    }
    __syncwarp();
  }
}

// (n, f) = I (w, v) for a packed spatial inertia about O: n = I_O w + h x v, f = m v - h x w
__device__ __forceinline__ void apply_inertia(const float* J, const float* w, const float* v, float* n, float* f) {
  float hv[3], hw[3];
  cross(J + 6, v, hv);
  cross(J + 6, w, hw);
  n[0] = J[0] * w[0] + J[3] * w[1] + J[4] * w[2] + hv[0];
  n[1] = J[3] * w[0] + J[1] * w[1] + J[5] * w[2] + hv[1];
  n[2] = J[4] * w[0] + J[5] * w[1] + J[2] * w[2] + hv[2];
  for (int k = 0; k < 3; k++) f[k] = J[9] * v[k] - hw[k];
}

// mass matrix rows (lane = dof: entries with its ancestor dofs) and qfrc_smooth = clamped actuator force - bias
__device__ __noinline__ void mass_and_force(World& s, int lane) {
  for (int e = lane; e < NTRIP / 4; e += 32) reinterpret_cast<float4*>(s.M)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  for (int i = lane; i < NV; i += 32) {
    const int b = ldi(g1_dof_body + i);
    const float w[3] = {s.dw[i][0], s.dw[i][1], s.dw[i][2]}, v[3] = {s.dv[i][0], s.dv[i][1], s.dv[i][2]};
    float J[10], n[3], f[3];
    for (int k = 0; k < 10; k++) J[k] = s.sm.I[b][k];
    apply_inertia(J, w, v, n, f);
    // ancestor dofs j < i (the dof's own body first for the free joint's dofs) and the diagonal
    unsigned long long anc = g1_body_dofmask[b] & ((1ull << i) - 1ull);
    while (anc) {
      const int j = __ffsll((long long)anc) - 1;
      anc &= anc - 1ull;
      s.M[TRI(i, j)] = dot3(s.dw[j], n) + dot3(s.dv[j], f);
    }
    s.M[TRI(i, i)] = dot3(w, n) + dot3(v, f) + ld(g1_dof_armature + i);
    // bias: the subtree wrench of the dof's body projected on its motion
    const float bias = dot3(w, s.sm.wr[b]) + dot3(v, s.sm.wr[b] + 3);
    float act = 0.f;
    bool clamp = false;
    if (i >= 6) {
      act = ld(g1_dof_kp + i) * (s.ctrl[i - 6] - s.qpos[i + 1]) - ld(g1_dof_kv + i) * s.qvel[i];
      const float lim = ld(g1_dof_frclim + i);
      act = fminf(fmaxf(act, -lim), lim);
      clamp = act <= -lim || act >= lim;
    }
    s.qsm[i] = act - bias;
    const unsigned bal = __ballot_sync(__activemask(), clamp);
    if (lane == 0) { if (i < 32) s.clamp_lo = bal; else s.clamp_hi = bal; }
  }
  __syncwarp();
}

// ---- dense Cholesky and solves --------------------------------------------------------------------------------
// chol_factor: A = L L' (then chol_solve: b <- A^-1 b), left-looking (Crout) in blocks of 4 columns, in shared
// memory, with compact code (rolled loops: a fully unrolled register factorisation is ~100 KB of instructions,
// beyond the instruction cache). Block k0: phase 1 forms for every row i >= k0 the dot products
// S_i^c = sum_{j<k0} L(i, j) L(c, j) for the block's columns c (lane l owns row k0 + l: its own row read once per j
// for all four columns, rows c as broadcasts); phase 2 finishes the block's columns one after another with the
// in-block terms (row c's entries from its lane by shuffle), the pivot from row c's lane, and L(i, c) =
// t_i / sqrt(pivot) (rsqrt refined by one Newton step; the inverse also goes to dinv for the solves). Block 0 covers
// rows 0..31; the tail rows 32..NV-1 get their block-0 entries right after it, one row per lane. A may alias L: A(i, c)
// is read by the lane owning row i when column c is finished, just before L(i, c) replaces it.
__device__ __forceinline__ float rsqrt_nr(float x) {
  float r = rsqrtf(x);
  return r * (1.5f - 0.5f * x * r * r);
}

constexpr int CB = 4;  // column block
constexpr int NT = NV - 32;  // tail rows 32 .. NV - 1, finished on lanes 0 .. NT - 1

__device__ __noinline__ void chol_factor(const float* A, float* L, float* dinv, int lane) {
  static_assert(NV > 32 && NT <= CB, "block 1 holds every row beyond 32");
  // Block k0 (columns k0 .. k0 + 3): lane l owns row r = k0 + l (rows k0 .. NV - 1 fit 32 lanes for k0 >= NT)
#pragma unroll 1
  for (int k0 = 0; k0 < NV; k0 += CB) {
    const int nb = min(CB, NV - k0);
    const int r = k0 + lane;  // this lane's row (valid when < NV)
    // phase 1: S[c] = sum_{j<k0} L(r, j) L(k0 + c, j)
    float S[CB] = {0.f, 0.f, 0.f, 0.f};
    if (r < NV && k0 > 0) {
      const float* Li = L + TRI(r, 0);
      const float* L0 = L + TRI(k0, 0);
      // k0 is a multiple of 4: four j at a time, their 20 loads issued together; row k0 + 1 starts k0 + 1 entries
      // after row k0, row k0 + 2 at 2 k0 + 3, row k0 + 3 at 3 k0 + 6 (rows past NV - 1 are not read)
      const float* L1 = L0 + (k0 + 1);
      const float* L2 = L0 + (2 * k0 + 3);
      const float* L3 = L0 + (3 * k0 + 6);
#pragma unroll 1
      for (int j = 0; j < k0; j += 4) {
        float li[4], a0[4], a1[4], a2[4], a3[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          li[q] = Li[j + q];
          a0[q] = L0[j + q];
          a1[q] = nb > 1 ? L1[j + q] : 0.f;
          a2[q] = nb > 2 ? L2[j + q] : 0.f;
          a3[q] = nb > 3 ? L3[j + q] : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
          S[0] += li[q] * a0[q];
          S[1] += li[q] * a1[q];
          S[2] += li[q] * a2[q];
          S[3] += li[q] * a3[q];
        }
      }
    }
    // phase 2: the block's columns in order; lane l keeps its row's new entries lo[c]
    float lo[CB] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < CB; c++) {
      if (c >= nb) break;
      const int col = k0 + c;
      float t0 = 0.f;
      if (r >= col && r < NV) t0 = A[TRI(r, col)] - S[c];
#pragma unroll
      for (int m = 0; m < c; m++) t0 -= lo[m] * __shfl_sync(FULL, lo[m], c);  // L(col, k0 + m): row col is lane c
      const float tkk = __shfl_sync(FULL, t0, c);
      const float inv = rsqrt_nr(fmaxf(tkk, 1e-30f));
      lo[c] = r > col ? t0 * inv : (r == col ? tkk * inv : 0.f);
      if (r >= col && r < NV) L[TRI(r, col)] = lo[c];
      if (lane == 0) dinv[col] = inv;
    }
    __syncwarp();
    // the tail rows' entries in block 0's columns: (A(32 + l, c) - sum_{q<c} L(32 + l, q) L(c, q)) / L(c, c)
    if (k0 == 0) {
      if (lane < NT) {
        float e[CB];
#pragma unroll
        for (int c = 0; c < CB; c++) {
          float v = A[TRI(32 + lane, c)];
#pragma unroll
          for (int q = 0; q < c; q++) v -= e[q] * L[TRI(c, q)];
          e[c] = v * dinv[c];
          L[TRI(32 + lane, c)] = e[c];
        }
      }
      __syncwarp();
    }
  }
}

// ---- the mass matrix's factor in tree-block order -------------------------------------------------------------
// The G1's dofs form five chains below the free root (dofs 0..5): left leg 6..11 and right leg 12..17 (children of
// the root), the waist 18..20, left arm 21..27 and right arm 28..34 (children of the waist's last body). M (and
// M + h kv) couples a dof only with its ancestors and descendants, so in the order legs, arms, waist, root (leaves
// first) its Cholesky factor keeps that pattern: each limb's block factors on its own (the four in parallel), which
// also gives the limb's columns of its ancestors' rows, and the 9 x 9 waist + root block factors last, after the
// limbs' products are subtracted (reference src/nablaengine/g1_engine/source.py CHOL_SOLVE and MuJoCo's mj_factorM,
// which use the same sparsity in reverse dof order). The factor is stored dense (packed lower triangle in that
// order, zeros outside the pattern), so chol_solve<true> solves with it on vectors in dof order.
__host__ __device__ constexpr int tb_dof(int p) { return p < 12 ? p + 6 : (p < 26 ? p + 9 : (p < 29 ? p - 8 : p - 29)); }
__host__ __device__ constexpr int tb_pos(int d) { return d < 6 ? d + 29 : (d < 18 ? d - 6 : (d < 21 ? d + 8 : d - 9)); }
static_assert(tb_pos(tb_dof(0)) == 0 && tb_pos(tb_dof(25)) == 25 && tb_pos(tb_dof(26)) == 26 &&
              tb_pos(tb_dof(34)) == 34 && tb_dof(12) == 21 && tb_dof(26) == 18 && tb_dof(29) == 0, "tree-block order");

// The factor's pattern in tree-block order: entry (p, q), p >= q, is structurally nonzero when p is in q's chain or
// in one of its ancestor chains (legs: the root; arms: the waist and the root; the waist: the root). The tape stores
// only these NTB entries of L_Q (packed-triangle order).
__host__ __device__ constexpr int tb_chain(int p) {  // left leg, right leg, left arm, right arm, waist, root
  return p < 6 ? 0 : (p < 12 ? 1 : (p < 19 ? 2 : (p < 26 ? 3 : (p < 29 ? 4 : 5))));
}
__host__ __device__ constexpr bool tb_nonzero(int p, int q) {
  const int a = tb_chain(p), b = tb_chain(q);
  return a == b || a == 5 || (a == 4 && (b == 2 || b == 3));
}
constexpr int tb_count() {
  int n = 0;
  for (int p = 0; p < NV; p++)
    for (int q = 0; q <= p; q++) n += tb_nonzero(p, q);
  return n;
}
constexpr int NTB = tb_count();
static_assert(NTB == 341 && NTB == NTB_TAPE, "the tree-block pattern of the G1");
struct TbIndex { unsigned short e[NTB]; };
constexpr TbIndex make_tb_index() {
  TbIndex t{};
  int n = 0;
  for (int p = 0; p < NV; p++)
    for (int q = 0; q <= p; q++)
      if (tb_nonzero(p, q)) t.e[n++] = (unsigned short)TRI(p, q);
  return t;
}
static __device__ const TbIndex g_tb_index = make_tb_index();

// right-looking elimination of N columns (positions cp0 .. cp0 + N - 1) on register rows: lane gb + li holds the
// row at position rowpos over those columns (the block's own rows first: lane gb + k is column k's row)
template <int N>
__device__ __forceinline__ void tb_rows(float (&a)[N], int li, int gb, bool act, int rowpos, int cp0, float* L,
                                        float* dinv) {
#pragma unroll
  for (int k = 0; k < N; k++) {
    const float piv = __shfl_sync(FULL, a[k], gb + k);
    const float inv = rsqrt_nr(fmaxf(piv, 1e-30f));
    const float l = a[k] * inv;  // L(row, column k); the pivot's own lane: sqrt(piv)
    if (act && li >= k) L[TRI(rowpos, cp0 + k)] = l;
    if (act && li == k) dinv[cp0 + k] = inv;
#pragma unroll
    for (int j = k + 1; j < N; j++) a[j] -= l * __shfl_sync(FULL, l, gb + j);
  }
}

// L L' = P (A + kv h diag(kv)) P' with A packed in dof order (the mass matrix), P the tree-block order; L and dinv in
// that order (L may not alias A)
__device__ __noinline__ void tb_factor(const float* A, bool kv, float* L, float* dinv, int lane) {
  const float h = G1_TIMESTEP;
  for (int e = lane; e < NTRIP / 4; e += 32) reinterpret_cast<float4*>(L)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  const int gb = lane & 16, li = lane - gb;
  {  // the arms (left on lanes 0..15, right on 16..31): the arm's 7 rows, then the waist's 3 and the root's 6
    const int first = gb ? 28 : 21;
    const int r = li < 7 ? first + li : (li < 10 ? 11 + li : li - 10);
    float a[7];
#pragma unroll
    for (int q = 0; q < 7; q++)
      a[q] = sym(A, r, first + q) + (kv && r == first + q ? h * ld(g1_dof_kv + r) : 0.f);
    tb_rows<7>(a, li, gb, true, tb_pos(r), tb_pos(first), L, dinv);
  }
  {  // the legs (left on lanes 0..11, right on 16..27): the leg's 6 rows, then the root's 6
    const int first = gb ? 12 : 6;
    const bool act = li < 12;
    const int r = li < 6 ? first + li : (act ? li - 6 : 0);
    float a[6];
#pragma unroll
    for (int q = 0; q < 6; q++)
      a[q] = act ? sym(A, r, first + q) + (kv && r == first + q ? h * ld(g1_dof_kv + r) : 0.f) : 0.f;
    tb_rows<6>(a, li, gb, act, tb_pos(r), tb_pos(first), L, dinv);
  }
  __syncwarp();
  // the waist + root block (positions 26..34) minus the limbs' products: entry (u, v), u >= v; the waist's rows hold
  // no leg columns (positions 0..11)
  for (int e = lane; e < 45; e += 32) {
    int u = (int)((sqrtf(8.f * e + 1.f) - 1.f) * 0.5f);
    if (TRI(u + 1, 0) <= e) u++;
    if (TRI(u, 0) > e) u--;
    const int v = e - TRI(u, 0), pu = 26 + u, pv = 26 + v, du = tb_dof(pu), dv = tb_dof(pv);
    const float* Lu = L + TRI(pu, 0);
    const float* Lv = L + TRI(pv, 0);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
    for (int c = u >= 3 && v >= 3 ? 0 : 12; c < 26; c += 2) {
      s0 += Lu[c] * Lv[c];
      s1 += Lu[c + 1] * Lv[c + 1];
    }
    L[TRI(pu, pv)] = sym(A, du, dv) + (kv && u == v ? h * ld(g1_dof_kv + du) : 0.f) - (s0 + s1);
  }
  __syncwarp();
  {  // the 9 x 9 block's factor on lanes 0..8
    const bool act = lane < 9;
    const int u = act ? lane : 0;
    float a[9];
#pragma unroll
    for (int q = 0; q < 9; q++) a[q] = L[TRI(26 + max(u, q), 26 + min(u, q))];
    __syncwarp();
    tb_rows<9>(a, lane, 0, act, 26 + u, 26, L, dinv);
  }
  __syncwarp();
}

// b <- (L L')^-1 b with the factor L and dinv = 1 / diag(L) in shared memory. Lane l keeps entry l (rows 0..31, the
// leading block, in blocks of 4: the block's 4 unknowns are solved redundantly on every lane from the block's
// diagonal entries (broadcast loads) and their current values (shuffles), then every other entry is updated with the
// block's 4 columns (forward: L(i, block), backward: L(block, i), read as rows); every lane keeps the NT tail rows
// 32..NV-1, solved after the leading block going forward (their sums over it by warp reductions) and before it going
// backward (their columns applied to every lane's entry)
// PERM: L is in tree-block order (tb_factor) and b in dof order: entry p of the solve is b[tb_dof(p)]
template <bool PERM = false>
__device__ __noinline__ void chol_solve(const float* L, const float* dinv, float* b, int lane) {
  static_assert(NV - NT == 32, "the leading block is one entry per lane");
  const int i0 = PERM ? tb_dof(lane) : lane;
  float y = b[i0], t[NT];
#pragma unroll
  for (int m = 0; m < NT; m++) t[m] = b[PERM ? tb_dof(32 + m) : 32 + m];
  __syncwarp();
#pragma unroll 1
  for (int k0 = 0; k0 < 32; k0 += CB) {
    float x[CB];
#pragma unroll
    for (int c = 0; c < CB; c++) x[c] = __shfl_sync(FULL, y, k0 + c);
#pragma unroll
    for (int c = 0; c < CB; c++) {
      float v = x[c];
#pragma unroll
      for (int m = 0; m < c; m++) v -= L[TRI(k0 + c, k0 + m)] * x[m];
      x[c] = v * dinv[k0 + c];
    }
#pragma unroll
    for (int c = 0; c < CB; c++) {
      if (lane == k0 + c) y = x[c];
      if (lane >= k0 + CB) y -= L[TRI(lane, k0 + c)] * x[c];
    }
  }
  // tail rows: t_m -= sum_{j<32} L(32 + m, j) y_j, then the NT x NT forward and backward substitutions
  float d[NT];
#pragma unroll
  for (int m = 0; m < NT; m++) d[m] = L[TRI(32 + m, lane)] * y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int m = 0; m < NT; m++) d[m] += __shfl_xor_sync(FULL, d[m], o);
#pragma unroll
  for (int m = 0; m < NT; m++) {
    float v = t[m] - d[m];
#pragma unroll
    for (int q = 0; q < m; q++) v -= L[TRI(32 + m, 32 + q)] * t[q];
    t[m] = v * dinv[32 + m];
  }
#pragma unroll
  for (int m = NT - 1; m >= 0; m--) {
    float v = t[m];
#pragma unroll
    for (int q = m + 1; q < NT; q++) v -= L[TRI(32 + q, 32 + m)] * t[q];
    t[m] = v * dinv[32 + m];
  }
#pragma unroll
  for (int m = 0; m < NT; m++) y -= L[TRI(32 + m, lane)] * t[m];
#pragma unroll 1
  for (int k0 = 32 - CB; k0 >= 0; k0 -= CB) {
    float x[CB];
#pragma unroll
    for (int c = 0; c < CB; c++) x[c] = __shfl_sync(FULL, y, k0 + c);
#pragma unroll
    for (int c = CB - 1; c >= 0; c--) {
      float v = x[c];
#pragma unroll
      for (int m = c + 1; m < CB; m++) v -= L[TRI(k0 + m, k0 + c)] * x[m];
      x[c] = v * dinv[k0 + c];
    }
#pragma unroll
    for (int c = 0; c < CB; c++) {
      if (lane == k0 + c) y = x[c];
      if (lane < k0) y -= L[TRI(k0 + c, lane)] * x[c];
    }
  }
  b[i0] = y;
#pragma unroll
  for (int m = 0; m < NT; m++)
    if (lane == m) b[PERM ? tb_dof(32 + m) : 32 + m] = t[m];
  __syncwarp();
}

// A v for A symmetric (packed lower triangle): lane l gets entry l in .x and, on lanes 0 .. NT - 1, entry 32 + l in
// .y (rows 0..31: one row per lane over all 35 columns; rows 32..34: split over the lanes, column j = lane, with the
// 3 x 3 tail block on lanes 0..2, and warp reductions)
__device__ __noinline__ float2 matvec(const float* A, const float* v, int lane) {
  float a0 = 0.f, a1 = 0.f;
#pragma unroll 6
  for (int j = 0; j < NV - 1; j += 2) {
    a0 += sym(A, lane, j) * v[j];
    a1 += sym(A, lane, j + 1) * v[j + 1];
  }
  if (NV & 1) a0 += A[TRI(NV - 1, lane)] * v[NV - 1];
  float t[NT];
#pragma unroll
  for (int m = 0; m < NT; m++) {
    t[m] = A[TRI(32 + m, lane)] * v[lane];
    if (lane < NT) t[m] += sym(A, 32 + m, 32 + lane) * v[32 + lane];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int m = 0; m < NT; m++) t[m] += __shfl_xor_sync(FULL, t[m], o);
  return make_float2(a0 + a1, lane == 0 ? t[0] : (lane == 1 ? t[1] : (lane == 2 ? t[2] : 0.f)));
}
// lane l's entries of a vector in matvec's layout: .x = v[l], .y = v[32 + l] on lanes 0 .. NT - 1 (else 0)
__device__ __forceinline__ float2 lanes_of(const float* v, int lane) {
  return make_float2(v[lane], lane < NT ? v[32 + lane] : 0.f);
}
__device__ __forceinline__ void store_lanes(float* v, float2 x, int lane) {
  v[lane] = x.x;
  if (lane < NT) v[32 + lane] = x.y;
}

// the dofs that move only body 1 (m1, Jacobian sign -1) / only body 2 (m2, sign +1) of contact pair pr
__device__ __forceinline__ void body_masks(unsigned bb, unsigned long long* m1, unsigned long long* m2) {
  const unsigned long long a = __ldg(g1_body_dofmask + (bb & 255u)), b = __ldg(g1_body_dofmask + (bb >> 8));
  *m1 = a & ~b;
  *m2 = b & ~a;
}

// contact c's frame rows: normal, tangent 1 (stored) and tangent 2 = normal x tangent 1 (both frames of the
// primitives, make_frame's and the capsule-plane axis frame, have that third row)
__device__ __forceinline__ void frame_rows(const World& s, int c, float* fr) {
#pragma unroll
  for (int k = 0; k < 6; k++) fr[k] = s.con_fr[c][k];
  cross(fr, fr + 3, fr + 6);
}

// ---- collision ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ void zaxis(const float* q, float* a) {
  const float ez[3] = {0.f, 0.f, 1.f};
  qrot(q, ez, a);
}
__device__ __forceinline__ void make_frame(const float* n, float* fr) {  // MuJoCo's make_frame: rows n, b, n x b
  float b[3] = {0.f, 0.f, 0.f};
  if (n[1] > -0.5f && n[1] < 0.5f) b[1] = 1.f; else b[2] = 1.f;
  const float d = dot3(n, b);
  for (int k = 0; k < 3; k++) b[k] -= n[k] * d;
  const float bn = sqrtf(dot3(b, b));
  if (bn > 0.f)
    for (int k = 0; k < 3; k++) b[k] /= bn;
  float c[3];
  cross(n, b, c);
  for (int k = 0; k < 3; k++) { fr[k] = n[k]; fr[3 + k] = b[k]; fr[6 + k] = c[k]; }
}
__device__ __forceinline__ void sphere_sphere(const float* p1, float r1, const float* p2, float r2, float* dist,
                                              float* pos, float* n) {
  const float dir[3] = {p2[0] - p1[0], p2[1] - p1[1], p2[2] - p1[2]};
  const float d = sqrtf(dot3(dir, dir));
  if (d == 0.f) { n[0] = 1.f; n[1] = 0.f; n[2] = 0.f; }
  else for (int k = 0; k < 3; k++) n[k] = dir[k] / d;
  *dist = d - (r1 + r2);
  const float hp = r1 + 0.5f * *dist;
  for (int k = 0; k < 3; k++) pos[k] = p1[k] + n[k] * hp;
}

// The bounding test of pair pr at the current geom poses (no contact at zero margin when it fails)
__device__ __forceinline__ bool bounding(const World& s, int pr) {
  const int g1 = ldi(g1_pair_g1 + pr), g2 = ldi(g1_pair_g2 + pr);
  const float dif[3] = {s.col.gx[g2][0] - s.col.gx[g1][0], s.col.gx[g2][1] - s.col.gx[g1][1],
                        s.col.gx[g2][2] - s.col.gx[g1][2]};
  if (ldi(g1_geom_type + g1) == 0) {
    float n[3];
    zaxis(s.col.gq[g1], n);
    return dot3(dif, n) <= ld(g1_geom_rbound + g2);
  }
  const float rb = ld(g1_geom_rbound + g1) + ld(g1_geom_rbound + g2);
  return dot3(dif, dif) <= rb * rb;
}

// up to two contacts of one candidate pair (slot, distance, point, frame rows), kept in registers until the warp's
// prefix sum gives their contact indices
struct Hit {
  int n, slot[2];
  float dist[2], pos[2][3], fr[2][6];  // frame rows: normal, tangent 1
};

// Narrow phase of candidate pair pr: its contacts (0..2, dist < 0) into h (h.n counted up from 0). MuJoCo Warp's
// primitives at margin 0.
__device__ __forceinline__ void collide(World& s, int pr, Hit& h, int* unsup) {
  const int g1 = ldi(g1_pair_g1 + pr), g2 = ldi(g1_pair_g2 + pr);
  const int t1 = ldi(g1_geom_type + g1), t2 = ldi(g1_geom_type + g2);
  float p1[3], p2[3];
  for (int k = 0; k < 3; k++) { p1[k] = s.col.gx[g1][k]; p2[k] = s.col.gx[g2][k]; }
  const float r1 = ld(g1_geom_size + 3 * g1), r2 = ld(g1_geom_size + 3 * g2);
  auto emit = [&](int slot, float dist, const float* pos, const float* fr) {
    if (h.n == 0) {
      h.slot[0] = slot; h.dist[0] = dist;
      for (int k = 0; k < 3; k++) h.pos[0][k] = pos[k];
      for (int k = 0; k < 6; k++) h.fr[0][k] = fr[k];
    } else {
      h.slot[1] = slot; h.dist[1] = dist;
      for (int k = 0; k < 3; k++) h.pos[1][k] = pos[k];
      for (int k = 0; k < 6; k++) h.fr[1][k] = fr[k];
    }
    h.n++;
  };
  if (t1 == 0) {  // plane (the floor) against a sphere or a capsule
    float nrm[3];
    zaxis(s.col.gq[g1], nrm);
    const float poff = dot3(p1, nrm);
    if (t2 == 2) {
      const float dist = dot3(p2, nrm) - poff - r2;
      if (dist < 0.f) {
        float pos[3], fr[9];
        const float hp = r2 + 0.5f * dist;
        for (int k = 0; k < 3; k++) pos[k] = p2[k] - nrm[k] * hp;
        make_frame(nrm, fr);
        emit(0, dist, pos, fr);
      }
    } else if (t2 == 3) {
      const float hl = ld(g1_geom_size + 3 * g2 + 1);
      float ax[3], fr[9];
      zaxis(s.col.gq[g2], ax);
      float d[2], ce[2][3];
      for (int e = 0; e < 2; e++) {
        for (int k = 0; k < 3; k++) ce[e][k] = e == 0 ? p2[k] + hl * ax[k] : p2[k] - hl * ax[k];
        d[e] = dot3(ce[e], nrm) - poff - r2;
      }
      if (d[0] < 0.f || d[1] < 0.f) {
        // frame: the capsule axis projected on the plane when that projection is long enough
        const float na = dot3(nrm, ax);
        float b[3] = {ax[0] - nrm[0] * na, ax[1] - nrm[1] * na, ax[2] - nrm[2] * na};
        const float bn = sqrtf(dot3(b, b));
        if (bn < 0.5f) make_frame(nrm, fr);
        else {
          for (int k = 0; k < 3; k++) b[k] /= bn;
          float c[3];
          cross(nrm, b, c);
          for (int k = 0; k < 3; k++) { fr[k] = nrm[k]; fr[3 + k] = b[k]; fr[6 + k] = c[k]; }
        }
        for (int e = 0; e < 2; e++)
          if (d[e] < 0.f) {
            float pos[3];
            const float hp = r2 + 0.5f * d[e];
            for (int k = 0; k < 3; k++) pos[k] = ce[e][k] - nrm[k] * hp;
            emit(e, d[e], pos, fr);
          }
      }
    } else {
      *unsup |= UNSUPPORTED_PAIR;
    }
    return;
  }
  if (t1 == 2 && t2 == 2) {  // sphere-sphere
    float dist, pos[3], nn[3], fr[9];
    sphere_sphere(p1, r1, p2, r2, &dist, pos, nn);
    if (dist < 0.f) { make_frame(nn, fr); emit(0, dist, pos, fr); }
    return;
  }
  if (t1 == 2 && t2 == 3) {  // sphere-capsule: the regularised closest point of the segment
    const float hl = ld(g1_geom_size + 3 * g2 + 1);
    float ax[3], a[3], ab[3], ap[3], pt[3];
    zaxis(s.col.gq[g2], ax);
    for (int k = 0; k < 3; k++) { a[k] = p2[k] - ax[k] * hl; ab[k] = 2.f * hl * ax[k]; ap[k] = p1[k] - a[k]; }
    const float gam = dot3(ab, ab) + 1e-6f;
    const float t = fminf(fmaxf(dot3(ap, ab) / gam, 0.f), 1.f);
    for (int k = 0; k < 3; k++) pt[k] = a[k] + t * ab[k];
    float dist, pos[3], nn[3], fr[9];
    sphere_sphere(p1, r1, pt, r2, &dist, pos, nn);
    if (dist < 0.f) { make_frame(nn, fr); emit(0, dist, pos, fr); }
    return;
  }
  if (t1 == 3 && t2 == 3) {  // capsule-capsule: closest points of the segments (clamp cascade)
    const float hl1 = ld(g1_geom_size + 3 * g1 + 1), hl2 = ld(g1_geom_size + 3 * g2 + 1);
    float a1[3], a2[3], df[3];
    zaxis(s.col.gq[g1], a1);
    zaxis(s.col.gq[g2], a2);
    for (int k = 0; k < 3; k++) { a1[k] *= hl1; a2[k] *= hl2; df[k] = p1[k] - p2[k]; }
    const float ma = dot3(a1, a1), mb = -dot3(a1, a2), mc = dot3(a2, a2), u = -dot3(a1, df), v = dot3(a2, df);
    const float det = ma * mc - mb * mb;
    auto at = [&](float x1, float x2, float* dist, float* pos, float* nn) {
      const float v1[3] = {p1[0] + a1[0] * x1, p1[1] + a1[1] * x1, p1[2] + a1[2] * x1};
      const float v2[3] = {p2[0] + a2[0] * x2, p2[1] + a2[1] * x2, p2[2] + a2[2] * x2};
      sphere_sphere(v1, r1, v2, r2, dist, pos, nn);
    };
    if (fabsf(det) >= 1e-15f) {
      float x1 = (mc * u - mb * v) / det, x2 = (ma * v - mb * u) / det;
      if (x1 > 1.f) { x1 = 1.f; x2 = (v - mb) / mc; }
      else if (x1 < -1.f) { x1 = -1.f; x2 = (v + mb) / mc; }
      if (x2 > 1.f || x2 < -1.f) {
        const bool hi = x2 > 1.f;
        x2 = hi ? 1.f : -1.f;
        x1 = fminf(fmaxf(hi ? (u - mb) / ma : (u + mb) / ma, -1.f), 1.f);
      }
      float dist, pos[3], nn[3], fr[9];
      at(x1, x2, &dist, pos, nn);
      if (dist < 0.f) { make_frame(nn, fr); emit(0, dist, pos, fr); }
    } else {  // parallel: the ends of one segment against the other, at most two touching candidates
      int cnt = 0;
      for (int e = 0; e < 4 && cnt < 2; e++) {
        float x1, x2;
        if (e < 2) {
          x1 = e == 0 ? 1.f : -1.f;
          x2 = fminf(fmaxf(e == 0 ? (v - mb) / mc : (v + mb) / mc, -1.f), 1.f);
        } else {
          x2 = e == 2 ? 1.f : -1.f;
          x1 = fminf(fmaxf(e == 2 ? (u - mb) / ma : (u + mb) / ma, -1.f), 1.f);
        }
        float dist, pos[3], nn[3], fr[9];
        at(x1, x2, &dist, pos, nn);
        if (dist <= 0.f) {
          cnt++;
          if (dist < 0.f) { make_frame(nn, fr); emit(e, dist, pos, fr); }
        }
      }
    }
    return;
  }
  *unsup |= UNSUPPORTED_PAIR;
  return;
}

// geom poses, broad phase (ballot-compacted candidates in pair order), narrow phase (each lane's contacts held in
// registers, a prefix sum over the warp, then written): contacts in pair order, deterministic
__device__ __noinline__ void collision(World& s, int lane) {
  for (int g = lane; g < NG; g += 32) {
    const int b = ldi(g1_geom_body + g);
    const float gp[3] = {ld(g1_geom_pos + 3 * g), ld(g1_geom_pos + 3 * g + 1), ld(g1_geom_pos + 3 * g + 2)};
    const float gq[4] = {ld(g1_geom_quat + 4 * g), ld(g1_geom_quat + 4 * g + 1), ld(g1_geom_quat + 4 * g + 2),
                         ld(g1_geom_quat + 4 * g + 3)};
    float t[3];
    qrot(s.Q[b], gp, t);
    for (int k = 0; k < 3; k++) s.col.gx[g][k] = s.X[b][k] + t[k];
    qmul(s.Q[b], gq, s.col.gq[g]);
  }
  __syncwarp();
  const unsigned below = (1u << lane) - 1u;
  int ncand = 0;
  for (int k = 0; k < (NP + 31) / 32; k++) {
    const int pr = lane + 32 * k;
    const bool keep = pr < NP && bounding(s, pr);
    const unsigned bal = __ballot_sync(FULL, keep);
    if (keep) s.col.cand[ncand + __popc(bal & below)] = (unsigned short)pr;
    ncand += __popc(bal);
  }
  __syncwarp();
  int total = 0, unsup = 0;
  for (int c0 = 0; c0 < ncand; c0 += 32) {
    const int ci = c0 + lane;
    const int pr = ci < ncand ? s.col.cand[ci] : -1;
    Hit h;
    h.n = 0;
    if (pr >= 0) collide(s, pr, h, &unsup);
    int incl = h.n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += t;
    }
    const int base = total + incl - h.n;
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int c = base + e;
      if (e >= h.n || c >= WCON) continue;
      s.con_pair[c] = pr;
      s.con_slot[c] = (unsigned char)h.slot[e];
      s.con_dist[c] = h.dist[e];
      for (int k = 0; k < 3; k++) s.con_pos[c][k] = h.pos[e][k];
      for (int k = 0; k < 6; k++) s.con_fr[c][k] = h.fr[e][k];
    }
    total += __shfl_sync(FULL, incl, 31);
  }
  unsup = (int)__reduce_or_sync(FULL, (unsigned)unsup);
  if (lane == 0) {
    s.ncand = ncand;
    s.ncon_raw = total;
    s.ncon = min(total, WCON);
    s.unsup |= unsup | (total > WCON ? CONTACT_OVERFLOW : 0);
  }
  __syncwarp();
}

// per contact: friction, the frame rows' moments about O and the support masks (lane = contact); then the groups:
// the contacts between the same two bodies (in contact order, numbered by their first contact), which share the
// support and the sign of every Jacobian column, so the Hessian and J' f treat a group as one spatial stiffness /
// one wrench
__device__ __noinline__ void contact_setup(World& s, int lane) {
  const int ncon = uni(s.ncon);
  const float O[3] = {s.O[0], s.O[1], s.O[2]};
  __syncwarp();
  for (int c = lane; c < ncon; c += 32) {
    const int pr = s.con_pair[c];
    // condim 1 (frictionless) contacts: mu = 0 makes the pyramid formulas below reduce to the normal row
    s.con_mu[c] = ldi(g1_pair_dim + pr) != 3 ? 0.f : (ldi(g1_pair_foot + pr) ? s.fric : ld(g1_pair_mu + pr));
    // the contact point relative to O (the frame rows' moments are (pos - O) x row)
    for (int k = 0; k < 3; k++) s.con_pos[c][k] -= O[k];
  }
  // group leaders: the first contact of each (body1, body2); the keys are kept in cs.g for a moment
  int ngroup = 0;
  for (int c0 = 0; c0 < ncon; c0 += 32) {
    const int c = c0 + lane;
    int key = -1 - lane, lead = c;
    if (c < ncon) {
      const int pr = s.con_pair[c];
      const int b1 = ldi(g1_geom_body + ldi(g1_pair_g1 + pr)), b2 = ldi(g1_geom_body + ldi(g1_pair_g2 + pr));
      s.con_bb[c] = (unsigned short)(b1 | b2 << 8);
      key = b1 * 32 + b2;
      for (int e = 0; e < c0; e++)  // an earlier chunk (only past 32 contacts)
        if (s.cs.g.key[e] == key) { lead = e; break; }
    }
    const unsigned same = __match_any_sync(FULL, key);
    if (lead == c) lead = c0 + __ffs(same) - 1;
    const bool leader = c < ncon && lead == c;
    const unsigned bal = __ballot_sync(FULL, leader);
    if (c < ncon) {
      s.cs.g.key[c] = key;
      s.cs.g.lead[c] = (unsigned char)lead;
      if (leader) s.cs.g.grp[c] = (unsigned char)(ngroup + __popc(bal & ((1u << lane) - 1u)));
    }
    ngroup += __popc(bal);
    __syncwarp();
  }
  for (int c = lane; c < ncon; c += 32) s.cs.g.grp[c] = s.cs.g.grp[s.cs.g.lead[c]];
  __syncwarp();
  // the member lists: group g's size (lane g), an exclusive prefix sum over the groups, then its members in order
  int carry = 0;
  for (int g0 = 0; g0 < ngroup; g0 += 32) {
    const int g = g0 + lane;
    int n = 0;
    if (g < ngroup)
      for (int c = 0; c < ncon; c++) n += s.cs.g.grp[c] == g;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += t;
    }
    if (g < ngroup) {
      int k = carry + incl - n;
      s.grp_first[g] = (unsigned char)k;
      for (int c = 0; c < ncon; c++)
        if (s.cs.g.grp[c] == g) s.grp_mem[k++] = (unsigned char)c;
    }
    carry += __shfl_sync(FULL, incl, 31);
  }
  if (lane == 0) { s.grp_first[ngroup] = (unsigned char)ncon; s.ngroup = ngroup; }
  __syncwarp();
}

// ---- constraint rows -----------------------------------------------------------------------------------------------
// J_d v of every contact's frame rows for the generalised vector v, into cs.jd. First the bodies' spatial motions at
// O (lane = body, kept in registers): its own contribution, the hinge's v_d (dw, dv), or for the root its 6 dofs
// (translations e_k, rotations about O), then the sums over the ancestors by pointer jumping (ceil(log2(depth + 1))
// = 4 rounds: add the value held by the current ancestor pointer, then jump the pointer; the world body holds 0 and
// points to itself). Then per contact (lane = contact) the two bodies' motions by shuffles from their lanes, and the
// relative velocity at the contact point along the frame rows.
__device__ __noinline__ void contact_jv(World& s, const float* v, int lane) {
  static_assert(MAXD < 16, "4 pointer-jumping rounds");
  float a[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int par = 0;
  if (lane == 1) {
    for (int k = 0; k < 3; k++) {
      a[3 + k] = v[k];
      a[k] = v[3] * s.dw[3][k] + v[4] * s.dw[4][k] + v[5] * s.dw[5][k];
    }
  } else if (lane >= 2 && lane < NB) {
    const int d = lane + 4;  // the hinge dof of body b >= 2 (dofs in body order)
    const float vd = v[d];
    for (int k = 0; k < 3; k++) { a[k] = vd * s.dw[d][k]; a[3 + k] = vd * s.dv[d][k]; }
    par = ldi(g1_body_parent + lane);
  }
#pragma unroll
  for (int round = 0; round < 4; round++) {
#pragma unroll
    for (int k = 0; k < 6; k++) a[k] += __shfl_sync(FULL, a[k], par);
    par = __shfl_sync(FULL, par, par);
  }
  const int ncon = uni(s.ncon);
  for (int c0 = 0; c0 < ncon; c0 += 32) {
    const int c = c0 + lane;
    const bool valid = c < ncon;
    const int bb = valid ? s.con_bb[c] : 0, b1 = bb & 255, b2 = bb >> 8;
    float dV[6];
#pragma unroll
    for (int k = 0; k < 6; k++) dV[k] = __shfl_sync(FULL, a[k], b2) - __shfl_sync(FULL, a[k], b1);
    if (valid) {
      // the relative velocity at the contact point: v_O + w x (pos - O); frame row d: row . that
      float u[3], fr[9];
      cross(dV, s.con_pos[c], u);
      for (int k = 0; k < 3; k++) u[k] += dV[3 + k];
      frame_rows(s, c, fr);
      for (int d = 0; d < 3; d++) s.cs.jd[c][d] = dot3(fr + 3 * d, u);
    }
  }
  __syncwarp();
}

// J v of every row into registers: row r = lane + 32 t into o[t], 0 past the row count (contact rows from cs.jd,
// limit rows from v)
__device__ __forceinline__ void rows_jv(World& s, const float* v, float (&o)[ROWS_PER_LANE], int lane) {
  contact_jv(s, v, lane);
  const int nefc = s.nefc;
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++) {
    const int r = lane + 32 * t;
    float val = 0.f;
    if (r < nefc) {
      const int kind = s.efc_kind[r], a = s.efc_a[r], b = s.efc_b[r];
      if (kind == ROW_LIMIT) val = b * v[a];
      else if (kind == ROW_PYRAMID) val = s.cs.jd[a][0] + ((b & 1) ? -1.f : 1.f) * s.con_mu[a] * s.cs.jd[a][1 + (b >> 1)];
      else val = s.cs.jd[a][0];
    }
    o[t] = val;
  }
  __syncwarp();
}

// refsafe impedance at the row position pos: stiffness k, damping b, impedance imp (solimp power 2 folded)
__device__ __noinline__ void impedance(const float* solref, const float* solimp, float pos, float h, float* k,
                                          float* b, float* imp) {
  const float tc = fmaxf(solref[0], 2.f * h), dr = solref[1];
  const float dmin = fminf(fmaxf(solimp[0], 1e-4f), 0.9999f), dmax = fminf(fmaxf(solimp[1], 1e-4f), 0.9999f);
  const float width = fmaxf(1e-15f, solimp[2]), mid = fminf(fmaxf(solimp[3], 1e-4f), 0.9999f);
  *k = 1.f / fmaxf(1e-15f, dmax * dmax * tc * tc * dr * dr);
  *b = 2.f / fmaxf(1e-15f, dmax * tc);
  const float x = fabsf(pos) / width;
  if (x >= 1.f) *imp = dmax;
  else if (x <= 0.f) *imp = dmin;
  else {
    // solimp power 2 on every row of the model (the generator checks it): x^2 / mid, 1 - (1 - x)^2 / (1 - mid)
    const float y = x <= mid ? x * x / mid : 1.f - (1.f - x) * (1.f - x) / (1.f - mid);
    *imp = fminf(fmaxf(dmin + y * (dmax - dmin), dmin), dmax);
  }
}

// constraint rows: hinge limits (dof order), then per contact 4 pyramid rows (condim 3) or 1 normal row
__device__ __noinline__ void make_rows(World& s, int lane) {
  const float h = G1_TIMESTEP;
  const unsigned below = (1u << lane) - 1u;
  int nlim = 0;
  unsigned long long lmask = 0ull;
  for (int i0 = 0; i0 < NV; i0 += 32) {
    const int i = i0 + lane;
    float dlo = 1.f, dhi = 1.f;
    if (i >= 6 && i < NV) {
      const float q = s.qpos[i + 1];
      dlo = q - ld(g1_dof_range + 2 * i);
      dhi = ld(g1_dof_range + 2 * i + 1) - q;
    }
    const bool on = fminf(dlo, dhi) < 0.f;
    const unsigned bal = __ballot_sync(FULL, on);
    lmask |= (unsigned long long)bal << i0;
    if (on) {
      const int r = nlim + __popc(bal & below);
      const float pos = fminf(dlo, dhi), sg = dlo < dhi ? 1.f : -1.f;
      const float sr[2] = {ld(g1_jnt_solref), ld(g1_jnt_solref + 1)};
      const float si[5] = {ld(g1_jnt_solimp), ld(g1_jnt_solimp + 1), ld(g1_jnt_solimp + 2), ld(g1_jnt_solimp + 3),
                           ld(g1_jnt_solimp + 4)};
      float k, b, imp;
      impedance(sr, si, pos, h, &k, &b, &imp);
      const float R = fmaxf(1e-15f, ld(g1_dof_invweight0 + i) * (1.f - imp) / imp);
      s.efc_kind[r] = ROW_LIMIT; s.efc_a[r] = (short)i; s.efc_b[r] = (signed char)sg;
      s.efc_D[r] = 1.f / R;
      s.efc_jar[r] = -b * (sg * s.qvel[i]) - k * imp * pos;  // aref until newton_begin
    }
    nlim += __popc(bal);
  }
  // contact rows need J qvel
  contact_jv(s, s.qvel, lane);
  const int ncon = uni(s.ncon);
  int r0 = nlim;
  for (int c0 = 0; c0 < ncon; c0 += 32) {
    const int c = c0 + lane;
    const bool valid = c < ncon;
    const int pr = valid ? s.con_pair[c] : 0;
    const int dim = valid ? ldi(g1_pair_dim + pr) : 0;
    const int want = valid ? (dim == 3 ? 4 : 1) : 0;
    int incl = want;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += t;
    }
    const int first = r0 + incl - want;
    if (valid) {
      const int nr = max(0, min(want, WROWS - first));
      s.con_row0[c] = (unsigned char)min(first, 255);
      s.con_nrow[c] = (unsigned char)nr;
      const float mu = s.con_mu[c];
      const int bb = s.con_bb[c], b1 = bb & 255, b2 = bb >> 8;
      float iw = ld(g1_body_invweight0 + b1) + ld(g1_body_invweight0 + b2);
      if (dim == 3) iw = (mu * mu * iw + iw) * 2.f * mu * mu / (float)G1_IMPRATIO;
      const float sr[2] = {ld(g1_pair_solref), ld(g1_pair_solref + 1)};
      const float si[5] = {ld(g1_pair_solimp), ld(g1_pair_solimp + 1), ld(g1_pair_solimp + 2),
                           ld(g1_pair_solimp + 3), ld(g1_pair_solimp + 4)};
      float k, b, imp;
      const float dist = s.con_dist[c];
      impedance(sr, si, dist, h, &k, &b, &imp);
      const float D = 1.f / fmaxf(1e-15f, iw * (1.f - imp) / imp);
      for (int t = 0; t < nr; t++) {
        const int r = first + t;
        const float vel = dim == 3 ? s.cs.jd[c][0] + ((t & 1) ? -1.f : 1.f) * mu * s.cs.jd[c][1 + (t >> 1)]
                                   : s.cs.jd[c][0];
        s.efc_kind[r] = dim == 3 ? ROW_PYRAMID : ROW_NORMAL;
        s.efc_a[r] = (short)c;
        s.efc_b[r] = (signed char)t;
        s.efc_D[r] = D;
        s.efc_jar[r] = -b * vel - k * imp * dist;  // aref until newton_begin
      }
    }
    r0 += __shfl_sync(FULL, incl, 31);
  }
  if (lane == 0) {
    s.nlim = nlim;
    s.lim_mask = lmask;
    s.nefc = min(r0, WROWS);
    if (r0 > WROWS) s.unsup |= ROW_OVERFLOW;
  }
  __syncwarp();
}

// ---- Newton solver -------------------------------------------------------------------------------------------------
// The constrained acceleration a minimises c(a) = 1/2 (a - a0)' M (a - a0) + sum_r s_r(J_r a - aref_r) with a0 =
// qacc_smooth and s_r(x) = 1/2 D_r x^2 for x < 0 (the row's quadratic zone), 0 else: MuJoCo's primal Newton method on
// the pyramidal cone (reference g1_engine/step.py:1969-2137). Its Gauss term's lane-wise part, 1/2 (M a - qfrc_smooth)
// (a - a0) (M a0 = qfrc_smooth), for a dof pair in matvec's layout; the rows' part for the lane's rows.
__device__ __forceinline__ float gauss_part(const World& s, float2 ma, float2 a, int lane) {
  float g = 0.5f * (ma.x - s.qsm[lane]) * (a.x - s.qacc0[lane]);
  if (lane < NT) g += 0.5f * (ma.y - s.qsm[32 + lane]) * (a.y - s.qacc0[32 + lane]);
  return g;
}
__device__ __forceinline__ float rows_part(const float (&x)[ROWS_PER_LANE], const float (&D)[ROWS_PER_LANE]) {
  float g = 0.f;
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++)
    if (x[t] < 0.f) g += 0.5f * D[t] * x[t] * x[t];
  return g;
}

// grad = M qacc - qfrc_smooth - J' f with f = -D jar on the active rows; returns |grad|. J' f: each contact's
// wrench at O from its rows' forces, summed per group (members in contact order), then per dof the groups whose
// support holds it (sign +1 on body 2's chain, -1 on body 1's) and the dof's limit row
__device__ __noinline__ float2 newton_grad(World& s, int lane, float extra) {
  const int ncon = uni(s.ncon), ngroup = uni(s.ngroup);
#pragma unroll 1
  for (int c = lane; c < ncon; c += 32) {
    const int r0 = s.con_row0[c], nr = s.con_nrow[c];
    float f[4];
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const float x = t < nr ? s.efc_jar[r0 + t] : 0.f;
      f[t] = x < 0.f ? -s.efc_D[r0 + t] * x : 0.f;
    }
    const float mu = s.con_mu[c];
    const float F[3] = {f[0] + f[1] + f[2] + f[3], mu * (f[0] - f[1]), mu * (f[2] - f[3])};
    float w[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, fr[9];
    frame_rows(s, c, fr);
    for (int d = 0; d < 3; d++)
      for (int k = 0; k < 3; k++) w[3 + k] += F[d] * fr[3 * d + k];
    cross(s.con_pos[c], w + 3, w);  // moment about O: (pos - O) x force
    for (int k = 0; k < 6; k++) s.cs.wr[c][k] = w[k];
  }
  __syncwarp();
  // group sums into the leader's slot: lane (g mod 5, entry) sums, then writes after a fence
#pragma unroll 1
  for (int g0 = 0; g0 < ngroup; g0 += 5) {
    const int g = g0 + lane / 6, e = lane % 6;
    float acc = 0.f;
    const bool on = lane < 30 && g < ngroup;
    if (on)
      for (int k = s.grp_first[g]; k < s.grp_first[g + 1]; k++) acc += s.cs.wr[s.grp_mem[k]][e];
    __syncwarp();
    if (on) s.cs.wr[s.grp_mem[s.grp_first[g]]][e] = acc;
    __syncwarp();
  }
  // lane l: dof 3 + l (dofs 3..34 in one pass); dofs 0..2 (the root translations, motion e_k) get the linear force
  // of the groups whose support holds them (every lane accumulates those three sums)
  const int i = lane + 3;
  float jtf = 0.f, ft[3] = {0.f, 0.f, 0.f};
  const unsigned long long lmask = s.lim_mask;  // the dof's limit row: its rank among the dofs with one
  const int lr = (lmask >> i) & 1ull ? __popcll(lmask & ((1ull << i) - 1ull)) : -1;
  if (lr >= 0) {
    const float x = s.efc_jar[lr];
    if (x < 0.f) jtf = s.efc_b[lr] * (-s.efc_D[lr] * x);
  }
  const float w[3] = {s.dw[i][0], s.dw[i][1], s.dw[i][2]}, v[3] = {s.dv[i][0], s.dv[i][1], s.dv[i][2]};
  const unsigned long long bit = 1ull << i;
#pragma unroll 1
  for (int g = 0; g < ngroup; g++) {
    const int c = s.grp_mem[s.grp_first[g]];  // the group's first contact holds its sum
    unsigned long long m1, m2;
    body_masks(s.con_bb[c], &m1, &m2);
    const float* W = s.cs.wr[c];
    const float sg = (m2 & bit) ? 1.f : ((m1 & bit) ? -1.f : 0.f);
    if (sg != 0.f) jtf += sg * (dot3(w, W) + dot3(v, W + 3));
    const float st = (m2 & 1ull) ? 1.f : ((m1 & 1ull) ? -1.f : 0.f);  // the root dofs: all on a chain or none
    for (int k = 0; k < 3; k++) ft[k] += st * W[3 + k];
  }
  const float g = s.Ma[i] - s.qsm[i] - jtf;
  s.grad[i] = g;
  float gn = g * g;
  if (lane < 3) {
    const float g0 = s.Ma[lane] - s.qsm[lane] - (lane == 0 ? ft[0] : (lane == 1 ? ft[1] : ft[2]));
    s.grad[lane] = g0;
    gn += g0 * g0;
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {  // |grad|^2 and the caller's sum (the new cost), one butterfly
    gn += __shfl_xor_sync(FULL, gn, o);
    extra += __shfl_xor_sync(FULL, extra, o);
  }
  return make_float2(sqrtf(gn), extra);
}

// One level of the transposing reduction of N values per lane across the warp: lanes with bit W of their index keep
// the upper M = ceil(N / 2) values (moved down), the others the lower M, each adding its partner's copy; after the
// levels W = 16, 8, 4, 2, 1 of 21 values (23 shuffles) lane l holds the warp sum of entry kred_slot(l) (or none: -1)
template <int N, int W>
__device__ __forceinline__ void kred_level(float* v, int lane) {
  constexpr int M = (N + 1) / 2;
  const bool up = lane & W;
#pragma unroll
  for (int i = 0; i < M; i++) {
    const float hi = M + i < N ? v[M + i] : 0.f;
    const float keep = up ? hi : v[i], send = up ? v[i] : hi;
    v[i] = keep + __shfl_xor_sync(FULL, send, W);
  }
}
__host__ __device__ constexpr int kred_slot(int l) {
  int base = 0, cnt = 21, n = 21;
  for (int w = 16; w >= 1; w >>= 1) {
    const int m = (n + 1) / 2;
    if (l & w) { base += m; cnt = cnt > m ? cnt - m : 0; } else { cnt = cnt < m ? cnt : m; }
    n = m;
  }
  return cnt >= 1 ? base : -1;
}
struct KSlotTable { signed char slot[32]; };
constexpr KSlotTable make_kslot_table() {
  KSlotTable t{};
  for (int l = 0; l < 32; l++) t.slot[l] = (signed char)kred_slot(l);
  return t;
}
static __device__ const KSlotTable g_kslot = make_kslot_table();
// support pair e (packed lower triangle of the support ranks) -> a | b << 8
struct PairTable { unsigned short ab[KDOF * (KDOF + 1) / 2]; };
constexpr PairTable make_pair_table() {
  PairTable t{};
  int e = 0;
  for (int a = 0; a < KDOF; a++)
    for (int b = 0; b <= a; b++) t.ab[e++] = (unsigned short)(a | b << 8);
  return t;
}
static __device__ const PairTable g_pair_ab = make_pair_table();

// H = M + J' D J over the quadratic rows, into s.L (lower triangle). A contact row with direction u (n +- mu t_k)
// at the point pos has J_r = a' S with a = ((pos - O) x u, u) and S the dofs' motion vectors about O, so a group of
// contacts (one body pair) adds S' K S with the 6 x 6 spatial stiffness K = sum D a a' over its quadratic rows, on
// the group's support with the columns' signs
__device__ __noinline__ void hessian(World& s, int lane) {
  const int ngroup = uni(s.ngroup);
  const int kslot = __ldg(g_kslot.slot + lane);
  for (int e = lane; e < NTRIP / 4; e += 32)
    reinterpret_cast<float4*>(s.L)[e] = reinterpret_cast<const float4*>(s.M)[e];
  __syncwarp();
  for (int r = lane; r < s.nlim; r += 32)  // one limit row per dof: distinct diagonal entries
    if (s.efc_jar[r] < 0.f) s.L[TRI(s.efc_a[r], s.efc_a[r])] += s.efc_D[r];
  __syncwarp();
  PROF(s, 26);
#ifdef NB_PROFILE
  bool xbranch = false;  // a group on two branches of the tree (H fills outside M's pattern)
#endif
  for (int g = 0; g < ngroup; g++) {
    const int first = s.grp_first[g], nmem = s.grp_first[g + 1] - first;
    // K = sum of D a a' over the group's quadratic rows, a = ((pos - O) x u, u) with u = n +- mu t_k the row's
    // direction: lane 4 m + t holds the 21 products (upper triangle of 6 x 6, row order) of row t of the group's
    // member m (eight members at a time), and a transposing reduction leaves entry kslot on each lane
    float v[21];
#pragma unroll
    for (int e = 0; e < 21; e++) v[e] = 0.f;
    bool any = false;
#pragma unroll 1
    for (int base = 0; base < nmem; base += 8) {
      const int m = base + (lane >> 2), t = lane & 3;
      const int c = m < nmem ? s.grp_mem[first + m] : -1;
      if (c < 0 || t >= s.con_nrow[c]) continue;
      const int r = s.con_row0[c] + t;
      if (!(s.efc_jar[r] < 0.f)) continue;
      const float D = s.efc_D[r], mu = ((t & 1) ? -1.f : 1.f) * s.con_mu[c];
      float f[9];
      frame_rows(s, c, f);
      const int k = 3 + 3 * (t >> 1);
      const float u[3] = {f[0] + mu * f[k], f[1] + mu * f[k + 1], f[2] + mu * f[k + 2]};
      float a[6];
      cross(s.con_pos[c], u, a);
      a[3] = u[0]; a[4] = u[1]; a[5] = u[2];
      int e = 0;
#pragma unroll
      for (int e1 = 0; e1 < 6; e1++) {
        const float da = D * a[e1];
#pragma unroll
        for (int e2 = e1; e2 < 6; e2++) v[e++] += da * a[e2];
      }
      any = true;
    }
    if (!__any_sync(FULL, any)) { PROF(s, 27); continue; }  // no quadratic row in the group
    kred_level<21, 16>(v, lane);
    kred_level<11, 8>(v, lane);
    kred_level<6, 4>(v, lane);
    kred_level<3, 2>(v, lane);
    kred_level<2, 1>(v, lane);
    if (kslot >= 0) s.hs.K[kslot] = v[0];
    __syncwarp();
    const int lead = s.grp_mem[first];
    unsigned long long m1, m2;
    body_masks(s.con_bb[lead], &m1, &m2);
    const unsigned long long sup = m1 | m2;
    PROF(s, 27);
#ifdef NB_PROFILE
    xbranch |= m1 != 0ull && m2 != 0ull;
#endif
    const int nsup = __popcll(sup);
    // P_k = K s_i for the support dofs i (rank k: the k-th set bit of the support), signed
    {
      const int k = lane;
      const unsigned slo = (unsigned)sup, shi = (unsigned)(sup >> 32);
      const int nlo = __popc(slo);
      if (k < nsup) {
        const int i = k < nlo ? (int)__fns(slo, 0, k + 1) : 32 + (int)__fns(shi, 0, k - nlo + 1);
        const float sg = ((m2 >> i) & 1ull) ? 1.f : -1.f;
        const float* K = s.hs.K;
        const float v[6] = {sg * s.dw[i][0], sg * s.dw[i][1], sg * s.dw[i][2], sg * s.dv[i][0], sg * s.dv[i][1],
                            sg * s.dv[i][2]};
        // K rows from the packed upper triangle
        float P[6];
#pragma unroll
        for (int r = 0; r < 6; r++) {
          float acc = 0.f;
#pragma unroll
          for (int q = 0; q < 6; q++) {
            const int lo = r < q ? r : q, hi = r < q ? q : r;
            acc += K[lo * 6 - lo * (lo - 1) / 2 + (hi - lo)] * v[q];
          }
          P[r] = acc;
        }
        for (int r = 0; r < 6; r++) s.hs.P[k][r] = P[r];
        s.hs.dof[k] = (unsigned char)i;
      }
    }
    __syncwarp();
    PROF(s, 28);
    // H(dof a, dof b) += (sign_a s_a) . P_b for the support pairs a >= b
    const int npair = nsup * (nsup + 1) / 2;
    PROF_COUNT(30, 1);
    PROF_COUNT(31, npair);
#pragma unroll 1
    for (int e = lane; e < npair; e += 32) {
      const unsigned ab = __ldg(g_pair_ab.ab + e);
      const int a = ab & 255u, b = ab >> 8;
      const int da = s.hs.dof[a], db = s.hs.dof[b];
      const float sa = ((m2 >> da) & 1ull) ? 1.f : -1.f;
      const float* P = s.hs.P[b];
      const float v = sa * (s.dw[da][0] * P[0] + s.dw[da][1] * P[1] + s.dw[da][2] * P[2] + s.dv[da][0] * P[3]
                            + s.dv[da][1] * P[4] + s.dv[da][2] * P[5]);
      s.L[TRI(da, db)] += v;
    }
    __syncwarp();
    PROF(s, 29);
  }
#ifdef NB_PROFILE
  PROF_COUNT(32, xbranch ? 1 : 0);
  PROF_COUNT(33, 1);
#endif
}

// The Newton start: of the two candidates, the warm start (qacc on entry) and a0 itself, the one with the lower cost
// (a tie takes a0); then its gradient. The rows' aref, left in efc_jar by make_rows, becomes J a - aref there. Then
// newton_iter runs one iteration at a time (Hessian and factor unless no row changed its zone, solve, exact line
// search, update, gradient, stopping test); the state between iterations (cost, count, converged, same zones) lives
// in the world record, so the caller can run the iterations of several worlds in lockstep.
__device__ __noinline__ void newton_begin(World& s, int lane) {
  // (values live across the calls below are kept few: what a call must preserve goes to the stack)
  const int nefc = uni(s.nefc);
  float x[ROWS_PER_LANE];
  auto minus_aref = [&]() {  // x = J a - aref, 0 past the rows
#pragma unroll
    for (int t = 0; t < ROWS_PER_LANE; t++) x[t] = lane + 32 * t < nefc ? x[t] - s.efc_jar[lane + 32 * t] : 0.f;
  };
  auto rows_cost = [&]() {
    float g = 0.f;
#pragma unroll
    for (int t = 0; t < ROWS_PER_LANE; t++) {
      const float D = lane + 32 * t < nefc ? s.efc_D[lane + 32 * t] : 0.f;
      if (x[t] < 0.f) g += 0.5f * D * x[t] * x[t];
    }
    return g;
  };
  // the warm start: its rows' J a - aref parked in L (free until the first Hessian)
  const float2 mw = matvec(s.M, s.qacc, lane);
  rows_jv(s, s.qacc, x, lane);
  minus_aref();
  const float cost_w = warp_sum(gauss_part(s, mw, lanes_of(s.qacc, lane), lane) + rows_cost());
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++) s.L[lane + 32 * t] = x[t];
  // a0: its Gauss term is 0 (a - a0 = 0); its M a0 is needed only when a0 is kept
  rows_jv(s, s.qacc0, x, lane);
  minus_aref();
  const float cost_0 = warp_sum(rows_cost());
  const bool warm = uall(cost_0 > cost_w);
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++)
    if (lane + 32 * t < nefc) s.efc_jar[lane + 32 * t] = warm ? s.L[lane + 32 * t] : x[t];
  if (!warm) store_lanes(s.qacc, lanes_of(s.qacc0, lane), lane);
  __syncwarp();
  store_lanes(s.Ma, warm ? mw : matvec(s.M, s.qacc0, lane), lane);
  if (lane == 0) { s.nls = 0; s.nfact = 0; }
  __syncwarp();
  newton_grad(s, lane, 0.f);
  if (lane == 0) { s.ncost = warm ? cost_w : cost_0; s.nit_cur = 0; s.ndone = 0; s.nsame = 0; }
  __syncwarp();
}

// The exact line search along the Newton direction p. On the ray a + alpha p the cost is a convex piecewise quadratic
// f(alpha) with slope f'(alpha) = a1 + alpha a2 + sum_{x_r + alpha j_r < 0} D_r j_r (x_r + alpha j_r) and curvature
// f''(alpha) = a2 + sum_{same rows} D_r j_r^2 (a1 = (M a - qfrc_smooth) . p, a2 = p' M p; x_r = J_r a - aref_r,
// j_r = J_r p). It is minimised by 1-D Newton steps kept inside a bracket of the minimiser, with the stopping rules
// of MuJoCo's exact line search as the reference applies them (reference g1_engine/step.py:2032-2084): no descent at
// alpha = 0; the slope below 1e-7 of its value at 0; a Newton step that stayed on its quadratic piece (the rows'
// zones the same at the new point: that point is the piece's, so the ray's, minimiser, found without evaluating the
// slope there); at most 40 slope evaluations. A Newton step outside the bracket is replaced by its midpoint, or by a
// doubling while no upper end is known.
struct LineSearchResult { float alpha; int evals; };
__device__ __forceinline__ LineSearchResult exact_line_search(const float (&x)[ROWS_PER_LANE],
                                                              const float (&j)[ROWS_PER_LANE],
                                                              const float (&D)[ROWS_PER_LANE], float a1, float a2) {
  float Dj[ROWS_PER_LANE], Djj[ROWS_PER_LANE];
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++) { Dj[t] = D[t] * j[t]; Djj[t] = Dj[t] * j[t]; }
  float alpha = 0.f, below = 0.f, above = 1e30f, slope0 = 0.f;
  unsigned zones_before = 0u;  // this lane's rows in the quadratic zone at the previous trial point (bit t)
  bool newton_step = false;    // the step to the current point was a Newton step inside the bracket
  int evals = 0;
  while (true) {
    unsigned zones = 0u;
    float fd = 0.f, fdd = 0.f;
#pragma unroll
    for (int t = 0; t < ROWS_PER_LANE; t++) {
      const float xt = x[t] + alpha * j[t];
      if (xt < 0.f) { zones |= 1u << t; fd += Dj[t] * xt; fdd += Djj[t]; }
    }
    if (__all_sync(FULL, newton_step && zones == zones_before)) break;  // landed on the piece's minimiser
    if (evals == 40) break;
    evals++;
    fd = warp_sum(fd) + a1 + alpha * a2;
    fdd = warp_sum(fdd) + a2;
    if (evals == 1) {
      slope0 = fd;
      if (uall(slope0 >= 0.f)) break;  // p is no descent direction: stay at alpha = 0
    }
    if (uall(fabsf(fd) <= 1e-7f * fabsf(slope0))) break;
    if (fd < 0.f) below = alpha; else above = alpha;
    float next = alpha - fd / fdd;
    newton_step = next > below && next < above;
    if (!newton_step) next = above < 1e29f ? 0.5f * (below + above) : 2.f * fmaxf(alpha, 1e-6f);
    zones_before = zones;
    alpha = next;
  }
  return {alpha, evals};
}

__device__ __noinline__ void newton_iter(World& s, int lane) {
  const float scale = 1.f / ((float)G1_MEANINERTIA * NV), tol = (float)G1_TOLERANCE;
  const float cost = s.ncost;
  PROF(s, 24);  // (profile builds: the wait at the block barrier before this iteration)
  if (uall(!s.nsame)) {  // (no row changed its zone in the last step: H and its factor in s.L are still exact)
    if (lane == 0) s.nfact++;
    hessian(s, lane);
    PROF(s, 7);
    chol_factor(s.L, s.L, s.dinv, lane);
    PROF(s, 8);
  }
  for (int i = lane; i < NV; i += 32) s.p[i] = -s.grad[i];
  __syncwarp();
  chol_solve(s.L, s.dinv, s.p, lane);
  PROF(s, 9);
  const int nefc = uni(s.nefc);
  const float2 mp = matvec(s.M, s.p, lane);
  float x[ROWS_PER_LANE], jp[ROWS_PER_LANE], D[ROWS_PER_LANE];
  rows_jv(s, s.p, jp, lane);
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++) {
    const int r = lane + 32 * t;
    x[t] = r < nefc ? s.efc_jar[r] : 0.f;
    D[t] = r < nefc ? s.efc_D[r] : 0.f;
  }
  const float2 p = lanes_of(s.p, lane), ma = lanes_of(s.Ma, lane);
  float a1 = (ma.x - s.qsm[lane]) * p.x, a2 = p.x * mp.x;
  if (lane < NT) { a1 += (ma.y - s.qsm[32 + lane]) * p.y; a2 += p.y * mp.y; }
  a1 = warp_sum(a1);
  a2 = warp_sum(a2);
  const LineSearchResult ls = exact_line_search(x, jp, D, a1, a2);
  const float alpha = ls.alpha;
  if (lane == 0) s.nls += ls.evals;
  PROF_COUNT(17, ls.evals);
  // the step: a, M a and the rows' J a - aref are linear in alpha; the new cost is summed with |grad|
  float2 a = lanes_of(s.qacc, lane);
  a.x += alpha * p.x; a.y += alpha * p.y;
  const float2 man = make_float2(ma.x + alpha * mp.x, ma.y + alpha * mp.y);
  store_lanes(s.qacc, a, lane);
  store_lanes(s.Ma, man, lane);
  float cpart = gauss_part(s, man, a, lane);
  bool chg = false;
#ifdef NB_PROFILE
  int nchg = 0;  // rows changing zone (profile builds: a histogram of them)
#endif
#pragma unroll
  for (int t = 0; t < ROWS_PER_LANE; t++) {
    const int r = lane + 32 * t;
    const float xn = x[t] + alpha * jp[t];
    chg |= (xn < 0.f) != (x[t] < 0.f);
#ifdef NB_PROFILE
    nchg += r < nefc && (xn < 0.f) != (x[t] < 0.f);
#endif
    if (xn < 0.f) cpart += 0.5f * D[t] * xn * xn;
    if (r < nefc) s.efc_jar[r] = xn;
  }
  const bool same_zones = !__any_sync(FULL, chg);
#ifdef NB_PROFILE
  {
    const int n = (int)__reduce_add_sync(FULL, (unsigned)nchg);
    const int slot = n == 0 ? 12 : (n <= 2 ? 13 : (n <= 4 ? 14 : (n <= 8 ? 15 : (n <= 16 ? 21 : 22))));
    if (slot != 12) PROF_COUNT(slot, 1);
    PROF_COUNT(23, n);
  }
#endif
  __syncwarp();
  PROF(s, 10);
  const float2 gc = newton_grad(s, lane, cpart);
  const float gn = gc.x, newcost = gc.y;
  const float improvement = scale * (cost - newcost);
  PROF(s, 11);
  PROF_COUNT(16, 1);
  if (lane == 0) {
    s.ncost = newcost;
    s.nit_cur++;
    s.nsame = same_zones;
    s.ndone = improvement < tol || scale * gn < tol;
  }
  __syncwarp();
}

// ---- one substep -------------------------------------------------------------------------------------------------
// stats: null, or this world's 8 counters of the substep (contacts kept, rows, Newton iterations, line-search
// evaluations, Hessian factorisations, broad-phase candidates, contacts found, 0), the inputs of the FLOP count
// substep_pre: smooth dynamics, qacc_smooth, collision, rows and the Newton start; substep_post: the work counters,
// implicitfast and the integration. Between them the caller runs newton_iter until the world is done.
__device__ __forceinline__ void tape_put(float* dst, const float* src, int n, int lane) {
  for (int i = lane; i < n; i += 32) __stcs(dst + i, src[i]);
}

__device__ __noinline__ void substep_pre(World& s, int lane, float* rec) {
  PROF_START(s);
  if (rec) {
    tape_put(rec + T_QPOS, s.qpos, NQ, lane);
    tape_put(rec + T_QVEL, s.qvel, NV, lane);
  }
  kinematics(s, lane);
  dof_motion(s, lane);
  PROF(s, 0);
  body_terms(s, lane);
  PROF(s, 1);
  mass_and_force(s, lane);
  PROF(s, 2);
  // qacc_smooth = M^-1 qfrc_smooth
  for (int i = lane; i < NV; i += 32) s.qacc0[i] = s.qsm[i];
  tb_factor(s.M, false, s.L, s.dinv, lane);
  chol_solve<true>(s.L, s.dinv, s.qacc0, lane);
  PROF(s, 3);
  collision(s, lane);
  PROF(s, 4);
  contact_setup(s, lane);
  make_rows(s, lane);
  PROF(s, 5);
  PROF_COUNT(18, s.ncon);
  PROF_COUNT(19, s.nefc);
  newton_begin(s, lane);
  PROF(s, 6);
}

// stats: null, or this world's 8 counters of the substep (contacts kept, rows, Newton iterations, line-search
// evaluations, Hessian factorisations, broad-phase candidates, contacts found, 0), the inputs of the FLOP count;
// rec: null or the tape record, full (REC_WORDS) or compact (REC_COMPACT: no L_Q)
__device__ __noinline__ void substep_post(World& s, int lane, int* stats, float* rec, bool full) {
  const float h = G1_TIMESTEP;
  PROF(s, 25);  // (profile builds: the wait at the block barriers after this world's last iteration)
  const int it = s.nit_cur;
  if (rec) {  // the Hessian factor at the final zones (re-assembled when the last step changed a zone or none ran)
    const bool refact = !s.nsame || it == 0;
    if (refact) {
      hessian(s, lane);
      chol_factor(s.L, s.L, s.dinv, lane);
    }
    tape_put(rec + T_LH, s.L, NTRI, lane);
    tape_put(rec + T_DINVH, s.dinv, NV, lane);
    bool sing = false;
    for (int i = lane; i < NV; i += 32) sing |= !(s.dinv[i] < 1e14f);
    sing = __any_sync(FULL, sing);
    tape_put(rec + T_ASTAR, s.qacc, NV, lane);
    const int ncon = s.ncon, nefc = s.nefc;
    for (int i = lane; i < MAXCON / 2; i += 32) {
      const unsigned e0 = 2 * i < ncon ? (unsigned)s.con_pair[2 * i] | (unsigned)s.con_slot[2 * i] << 9 : 0xffffu;
      const unsigned e1 = 2 * i + 1 < ncon ? (unsigned)s.con_pair[2 * i + 1] | (unsigned)s.con_slot[2 * i + 1] << 9
                                          : 0xffffu;
      __stcs(rec + T_CON + i, __uint_as_float(e0 | e1 << 16));
    }
    for (int r0 = 0; r0 < NEFC; r0 += 32) {
      const int r = r0 + lane;
      const unsigned z = __ballot_sync(FULL, r < nefc && s.efc_jar[r] < 0.f);
      if (lane == 0) __stcs(rec + T_ZONE + r0 / 32, __uint_as_float(z));
    }
    if (lane == 0) {
      __stcs(rec + T_CLAMP, __uint_as_float(s.clamp_lo));
      __stcs(rec + T_CLAMP + 1, __uint_as_float(s.clamp_hi));
      __stcs(rec + T_HDR, __uint_as_float((unsigned)ncon | (unsigned)nefc << 8 | (unsigned)s.nlim << 16));
      __stcs(rec + T_FLAGS, __uint_as_float((unsigned)s.unsup | (refact ? TAPE_REFACT : 0u) |
                                            (s.ndone ? 0u : TAPE_NONCONV) | (sing ? TAPE_SINGULAR : 0u)));
    }
    __syncwarp();
  }
  if (stats && lane == 0) {
    stats[0] = s.ncon; stats[1] = s.nefc; stats[2] = it; stats[3] = s.nls;
    stats[4] = s.nfact; stats[5] = s.ncand; stats[6] = s.ncon_raw; stats[7] = 0;
  }
  // implicitfast: (M + h kv) a_adv = M qacc; qvel += h a_adv; qpos integrated with the new qvel
  for (int i = lane; i < NV; i += 32) s.p[i] = s.Ma[i];
  __syncwarp();
  tb_factor(s.M, true, s.L, s.dinv, lane);
  chol_solve<true>(s.L, s.dinv, s.p, lane);
  if (rec) {
    if (full) {
      for (int e = lane; e < NTB; e += 32) __stcs(rec + T_LQ + e, s.L[g_tb_index.e[e]]);
      tape_put(rec + T_DINVQ, s.dinv, NV, lane);
    }
    tape_put(rec + T_AADV, s.p, NV, lane);
  }
  for (int i = lane; i < NV; i += 32) s.qvel[i] += h * s.p[i];
  __syncwarp();
  if (lane == 0) {
    s.nit = it;
    for (int k = 0; k < 3; k++) s.qpos[k] += h * s.qvel[k];
    const float w[3] = {s.qvel[3], s.qvel[4], s.qvel[5]};
    const float nw = sqrtf(dot3(w, w));
    if (nw > 0.f) {
      float sa, ca;
      sincosf(0.5f * h * nw, &sa, &ca);
      const float dq[4] = {ca, sa * w[0] / nw, sa * w[1] / nw, sa * w[2] / nw};
      const float q[4] = {s.qpos[3], s.qpos[4], s.qpos[5], s.qpos[6]};
      float o[4];
      qmul(q, dq, o);
      const float on = sqrtf(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      for (int k = 0; k < 4; k++) s.qpos[3 + k] = o[k] / on;
    }
  }
  for (int i = 6 + lane; i < NV; i += 32) s.qpos[i + 1] += h * s.qvel[i];
  __syncwarp();
  PROF(s, 12);
  PROF_COUNT(20, 1);
}

}  // namespace nbg1
