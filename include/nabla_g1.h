/* nabla_g1.h — C ABI of the B200 (sm_100a) batched Unitree G1 physics step (libnabla_g1.so).
 *
 * The drop-in boundary for the reference's "one control step of B independent G1 worlds" path. Every entry point is
 * plain C: device pointers, sizes and a CUDA stream; no torch or XLA types. All arrays are row-major, contiguous,
 * float32 (info: int32), on the device that is current when the function is called; the caller owns every buffer.
 * Launches are asynchronous on `stream` (no host synchronisation), so the calls can be captured in a CUDA graph
 * after nb_g1_upload has run once on the device. Each returns a cudaError_t value as int (0 = success).
 *
 * Shapes (mjlab G1): nq 36, nv 35, nu 29; B worlds. qpos (B,36): root position, root quaternion (w x y z), 29 hinge
 * angles; qvel (B,35): root linear velocity (world), root angular velocity (local frame), 29 hinge rates; warm (B,35):
 * the Newton warm start (the previous step's warm'); ctrl (B,29): PD setpoints; friction (B,): the 14 sole-floor
 * pairs' sliding friction; com (B,3): the torso's COM offset in its frame (m).
 */
#ifndef NABLA_G1_H
#define NABLA_G1_H

#ifdef __cplusplus
extern "C" {
#endif

#ifndef __CUDA_RUNTIME_API_H__
typedef struct CUstream_st* cudaStream_t;
#endif

/* Sizes compiled into the library, in this order: nq, nv, nu, nbody, maxcon (64), nefc (192), tape words per world
 * and substep, ABI version. Replaces the reference's `<pfx>_sizes(long long*)` (src/nablaengine/jax_ffi.py:255),
 * which the bindings check against their own constants before the first call. */
void nb_g1_sizes(long long out[8]);

/* Scratch bytes nb_g1_forward takes for nw worlds (16-byte aligned, caller-allocated, e.g. a torch uint8 tensor or
 * XLA's scratch allocator): the order in which the kernel's blocks take the worlds, 4 bytes per world rounded up to
 * 16; -1 for nw < 0. Replaces `long long <pfx>_work_bytes(int nw)` (src/nablaengine/jax_ffi.py:265), whose work
 * memory holds the split forward's hand-over records and its row-count ordering (g1_engine/host.py:229-301). */
long long nb_g1_work_bytes(int nw);

/* Per-device preparation: must run once on each device before its first step and before any stream capture (it
 * may synchronise the stream once). consts may be NULL: the mjlab G1 constants are compiled into the library.
 * Replaces `int <pfx>_upload(const float* consts, cudaStream_t)` (src/nablaengine/jax_ffi.py:214-227). */
int nb_g1_upload(const float* consts, cudaStream_t stream);

/* One control step of nw worlds: nsub substeps (1..32) of 5 ms, Newton capped at `iterations` (>= 0) per substep.
 * Outputs qpos' (B,36), qvel' (B,35), warm' (B,35) (the last substep's constraint solution), info (B,4) int32 =
 * [Newton iterations of the last substep, contacts the last substep's collision found (may exceed 64), constraint
 * rows of the last substep (<= 192), bits 1 unsupported geom pair / 4 contacts beyond 64 dropped / 16 rows beyond
 * 192 dropped, ORed over the substeps]. ocon (B,64,8) may be NULL: the last substep's contacts as (pair, dist,
 * pos[3], normal[3]), pair -1 past the count. tape (B, nsub, tape words) may be NULL: else the per-substep records
 * nb_g1_adjoint reads (the substep's input state, a*, a_adv, the Cholesky factor of the Newton Hessian, the contact
 * table, the constraint zones, the actuator clamp masks, flags, then the factor of M + h kv; nb_g1_forward_ex below
 * writes the compact record without the last); the outputs are bitwise the
 * same with and without it. work: nb_g1_work_bytes(nw) bytes, overwritten, or NULL: with it the worlds are first
 * sorted by root height (lowest first, a small kernel before the step) so that worlds of similar cost share a
 * block; without it they run in index order, slower; the outputs are bitwise the same either way. nw == 0 is a
 * no-op.
 * Replaces `int <pfx>_forward(cudaStream_t, int nw, ...)` (src/nablaengine/jax_ffi.py:266-279). */
int nb_g1_forward(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                  const float* ctrl, const float* friction, const float* com, int iterations, int nsub, float* qpos_out,
                  float* qvel_out, float* warm_out, int* info, float* ocon, float* tape, void* work);

/* The adjoint of one control step from its tape: the VJP of (qpos', qvel') with cotangents gq_out (B,36) (qpos form)
 * and gv_out (B,35), written to gq_in (B,36) (qpos form: root position, 2 xi (x) (0, tangent cotangent) for the root
 * quaternion xi, hinges), gv_in (B,35) and gctrl (B,29); info (B,) int32: flags of the replay (bit 13: the replayed
 * constraint rows differ from the forward's). tape: nb_g1_forward's tape of the same nw worlds and nsub substeps;
 * friction, com: that call's. clamp_kv: 0 (the actuator damping term kept on clamped dofs), 1 (exact), 2 (the soft
 * clamp with width clamp_soft; ctrl (B,29), that call's setpoints, required); ctrl is ignored otherwise (may be NULL).
 * normal: the self-contact normal derivative, 0 exact, 1 frozen, 2 regularised below 1e-3 m, 3 frozen below 1e-3 m.
 * Replaces `int <pfx>_adjoint(cudaStream_t, int nw, int nsub, tape, fric, com, gq_out, gv_out, gq_in, gv_in, gctrl,
 * info, ctrl, clamp_soft)` (src/nablaengine/jax_ffi.py:228-241), where clamp_kv and normal select one of 12 compiled
 * libraries; here they are the two trailing arguments of one entry. */
int nb_g1_adjoint(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction, const float* com,
                  const float* gq_out, const float* gv_out, float* gq_in, float* gv_in, float* gctrl, int* info,
                  const float* ctrl, float clamp_soft, int clamp_kv, int normal);

/* The full step Jacobian from a tape: jac (B,71,99) float32, row r = d(output r) / d(inputs) with the outputs
 * qpos' (36, qpos form) then qvel' (35) and the inputs in the tangent basis: qpos tangent (35: root position, root
 * rotation vector in the local frame, hinges), qvel (35), ctrl (29); info (B,) int32: the replay flags ORed over the
 * rows. Arguments otherwise as nb_g1_adjoint; one launch (one block per world, one lane per tangent-basis cotangent
 * of the output). No counterpart in the reference's ABI: its Jacobian is 71 calls of `<pfx>_adjoint` with unit
 * cotangents plus the qpos-to-tangent map (scripts/paper_bench/ours.py:99-110, benchmarks/bench/adapters/base.py:
 * 254-277); row r here equals that row within float32 rounding (the same VJP, its operations in another order). */
int nb_g1_jacobian(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction, const float* com,
                   float* jac, int* info, const float* ctrl, float clamp_soft, int clamp_kv, int normal);

/* The kinematics outputs of nw states (qpos (B,36), qvel (B,35), com (B,3)): qpos_n (B,36) (the root quaternion
 * normalised), xpos (B,31,3) and xquat (B,31,4) (body frames, the world body included), cvel (B,31,6) ([angular;
 * linear] twist of each body at the root's subtree COM), subtree_com (B,31,3). Replaces `<pfx>_kinematics`
 * (src/nablaengine/jax_ffi.py:281-286; semantics src/nablaengine/g1_engine/kinematics.py:1-47). */
int nb_g1_kinematics(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* com,
                     float* qpos_n, float* xpos, float* xquat, float* cvel, float* subtree_com);

/* Their VJP: the cotangents of the five outputs (same layouts) -> gq (B,36) (qpos form) and gv (B,35) of (qpos, qvel);
 * gq_in / gv_in (may be NULL) are added last (a step's outputs' own cotangents). com gets no gradient. Replaces
 * `<pfx>_kinematics_vjp` (src/nablaengine/jax_ffi.py:287-292). */
int nb_g1_kinematics_vjp(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* com,
                         const float* g_qpos_n, const float* g_xpos, const float* g_xquat, const float* g_cvel,
                         const float* g_subtree_com, const float* gq_in, const float* gv_in, float* gq, float* gv);

/* Diagnostics: device counters (unsigned long long, nb_g1_diag_count() of them, the caller's zero-initialised array,
 * added to by every call): forward calls, worlds, worlds with unsupported / overflow bits, worlds at the iteration
 * limit, tape records, records refactored / not converged / with a clamped pivot; backward calls, rows, rows with a
 * non-finite gradient (all / qpos / qvel / ctrl), rows with a non-finite cotangent, worlds with a replay mismatch; then
 * contact-overflow and row-overflow worlds. nb_g1_diag_backward also ORs the non-finite bits (1 qpos, 2 qvel, 4 ctrl,
 * 8 cotangent) << 16 into the backward's info. One small kernel each, stream-ordered after the call it counts.
 * Replaces the reference's counter kernels `k_diag_fwd` / `k_diag_bwd` (src/nablaengine/jax_ffi.py:334-425,
 * src/nablaengine/torch_ffi.py:101-157). */
long long nb_g1_diag_count(void);
int nb_g1_diag_forward(cudaStream_t stream, unsigned long long* counters, int nw, int nsub, int iterations,
                       const int* info, const float* tape);
int nb_g1_diag_backward(cudaStream_t stream, unsigned long long* counters, int nw, const float* gq, const float* gv,
                        const float* gctrl, const float* gq_out, const float* gv_out, int* info);

/* The record of one forward call, from that call's info (B,4): rec[4] (device memory, uint32) = [worlds, contacts
 * summed over the worlds, the most contacts of one world, the most constraint rows of one world], info's counts being
 * the last substep's; rec2 (may be NULL) receives a copy (e.g. the record kept per batch size). One small kernel,
 * stream-ordered after the forward it reads; the sum is kept modulo 2^32. Replaces the reference's last-forward record
 * `k_last_fwd` / `k_last_read` and its slots per batch size (src/nablaengine/jax_ffi.py:352-425, `last_forward`
 * :1487), which it keeps in the library; here the caller owns the record's memory. */
int nb_g1_last_forward(cudaStream_t stream, int nw, const int* info, unsigned* rec, unsigned* rec2);

/* The launch shapes on device dev (after nb_g1_upload on it): out[8] = [the forward's dynamic shared memory per
 * block (bytes), the forward's resident worlds per SM, the adjoint's shared memory per block, its resident worlds per
 * SM, the Jacobian's shared memory per block, its resident cotangents (Jacobian rows in flight) per SM, the device's
 * SM count, 0]; a world or row count of 0 means the kernel does not fit the device. Restores the caller's current device. Replaces
 * `int <pfx>_launch(int dev, long long* o)` (src/nablaengine/jax_ffi.py:243-253: the adjoint's shared memory and
 * resident worlds per SM). */
int nb_g1_launch(int dev, long long out[8]);

/* nb_g1_forward plus the per-substep work counters stats (B, nsub, 8) int32: contacts kept, constraint rows, Newton
 * iterations, line-search evaluations, Hessian factorisations, broad-phase candidate pairs, contacts found, 0; the
 * outputs are bitwise those of nb_g1_forward. The counters feed the
 * FLOP count of a step (the roofline of the benchmark). No counterpart in the reference's ABI: it exposes the same
 * counts through its debug profile build (src/nablaengine/g1_engine/step.py:44-53 PROF_PHASES). */
int nb_g1_forward_stats(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                        const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                        float* qpos_out, float* qvel_out, float* warm_out, int* info, int* stats);

/* The largest nw nb_g1_forward_noalloc accepts. */
#define NB_G1_NOALLOC_MAX_WORLDS 262144

/* nb_g1_forward for callers that cannot allocate device memory: code that runs where cudaMalloc is not allowed or
 * not wanted (inside a host callback, on a memory budget fixed in advance, or in a runtime whose allocator the caller
 * does not own). Same arguments, outputs and errors as nb_g1_forward without the work pointer, and bitwise the same
 * outputs. The world order that nb_g1_forward keeps in the caller's work memory lives here in one buffer inside the
 * library: NB_G1_NOALLOC_MAX_WORLDS int32 (1 MiB) that every device which loads the library holds until the process
 * exits. nw above NB_G1_NOALLOC_MAX_WORLDS returns cudaErrorInvalidValue (1) and launches nothing. The first call on
 * a device (the current device) looks up that device's copy of the buffer (cudaGetSymbolAddress, once per device):
 * make that first call before any stream capture. The address is kept for the rest of the process: cudaDeviceReset
 * on a device destroys its context and the buffer with it, and the kept address then points at nothing, so after a
 * reset of a device do not call nb_g1_forward_noalloc on it again in the same process. Every call on a device shares the buffer: the order of one call is
 * overwritten by the next (nothing in it needs to start at zero), so calls whose kernels overlap on the GPU, on
 * different streams, race on it and must be serialised by the caller. The call allocates and frees nothing.
 * No counterpart in the reference's ABI. */
int nb_g1_forward_noalloc(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                          const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                          float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape);

/* The compact tape. nb_g1_tape_words(0) = the full record (the tape words of nb_g1_sizes, 1224), (1) = the compact
 * record (848: the full record's first words, without the factor of M + h kv and its inverse diagonal, which the
 * adjoint and the Jacobian then rebuild from the replayed poses: 31 % less tape, the reader's work grows by the
 * rebuild). The _ex entries are nb_g1_forward / _adjoint / _jacobian / _diag_forward with the tape's record size
 * (one of those two values) as a last argument; the plain entries take full records. Anything else returns
 * cudaErrorInvalidValue. Outputs of the forward are bitwise the same for either record; the adjoint and the
 * Jacobian from compact records equal those from full ones within float32 rounding. No counterpart in the
 * reference's ABI (its tape is one fixed record, src/nablaengine/g1_engine/tape.py:27-43). */
long long nb_g1_tape_words(int compact);
int nb_g1_forward_ex(cudaStream_t stream, int nw, const float* qpos, const float* qvel, const float* warm,
                     const float* ctrl, const float* friction, const float* com, int iterations, int nsub,
                     float* qpos_out, float* qvel_out, float* warm_out, int* info, float* ocon, float* tape,
                     void* work, int tape_words);
int nb_g1_adjoint_ex(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction,
                     const float* com, const float* gq_out, const float* gv_out, float* gq_in, float* gv_in,
                     float* gctrl, int* info, const float* ctrl, float clamp_soft, int clamp_kv, int normal,
                     int tape_words);
int nb_g1_jacobian_ex(cudaStream_t stream, int nw, int nsub, const float* tape, const float* friction,
                      const float* com, float* jac, int* info, const float* ctrl, float clamp_soft, int clamp_kv,
                      int normal, int tape_words);
int nb_g1_diag_forward_ex(cudaStream_t stream, unsigned long long* counters, int nw, int nsub, int iterations,
                          const int* info, const float* tape, int tape_words);

#ifdef __cplusplus
}
#endif
#endif /* NABLA_G1_H */
