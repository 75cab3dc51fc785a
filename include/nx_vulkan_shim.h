/* nx_vulkan_shim.h -- the flat nxv_* C ABI of nx_vulkan, implemented for
 * NVIDIA B200 (sm_100a) in libnxv_b200.so.
 *
 * Drop-in contract: every function the reference declares in
 * c_src/nx_vulkan_shim.h:20-280 (and that its Rust NIF binds in
 * native/nx_vulkan_native/src/lib.rs:30-295) is exported here with the
 * identical name and signature, so the reference's NIF links against this
 * library unchanged.  Semantics kept from the reference:
 *
 *   - Handles are opaque void* to a buffer record that carries its byte
 *     size (c_src/nx_vulkan_shim.cpp:169-191).  Output buffers are
 *     allocated by the caller with nxv_buf_alloc before the op is called.
 *   - Every compute call takes a trailing `spv_path`.  Its basename picks the
 *     kernel family exactly as the reference's shader file did, e.g.
 *     "elementwise_binary_f64.spv" selects the f64 binary kernel through
 *     nxv_apply_binary (lib.rs:966-1001 reuses nxv_apply_binary for f64).
 *     The directory part is ignored.  An unknown basename returns -2.
 *   - Return codes: 0 ok, -1 null argument, -2 kernel unavailable for this
 *     spv basename (shim.cpp:257-260).  This library adds -3 invalid
 *     argument (size, op or shape out of range), -4 CUDA error, -5 not
 *     initialised.  Unlike the reference (shim.cpp:292-437, 931-994), no
 *     path ignores an error.
 *   - Ordering: all work for a device runs in order on one CUDA stream, so
 *     a result is valid for every later nxv_* call the moment the call
 *     returns (the reference waited on a fence per dispatch,
 *     Backend_par_vulkan.cpp:225-238).  Calls that hand data to the host
 *     (nxv_buf_download, nxv_reduce*, nxv_pool_clear, nxv_synchronize)
 *     wait for the stream.  NXV_SYNC=1 in the environment makes every call
 *     wait, which surfaces asynchronous kernel faults at the faulting call.
 *   - Thread safety: every entry point may be called from any thread; the
 *     buffer pool has its own lock.  There is no global submit lock
 *     (lib.rs:303-319 needed one for the shared VkQueue).
 */
#ifndef NX_VULKAN_SHIM_H
#define NX_VULKAN_SHIM_H

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Lifecycle (reference c_src/nx_vulkan_shim.h:20-27) ---------------- */

/* Select device 0 (or the devices named by NXV_DEVICES, comma-separated),
 * create its stream and memory pool.  Idempotent.  0 on success, non-zero
 * when no CUDA device is usable.  Replaces shim.h:22-24. */
int nxv_init(void);

/* Free pooled buffers, streams and per-device state.  Idempotent.
 * Replaces shim.h:26-27. */
void nxv_destroy(void);

/* ---- Introspection (shim.h:29-36) -------------------------------------- */

/* Name of the current device, valid until nxv_destroy; NULL before init.
 * Replaces shim.h:31-33. */
const char* nxv_device_name(void);

/* 1 when the device computes in f64 (always, on B200).  Replaces shim.h:35-36. */
int nxv_has_f64(void);

/* ---- Buffers and pool (shim.h:42-65) ----------------------------------- */

/* Device buffer of n_bytes from the exact-size pool (hit) or the device's
 * stream-ordered cudaMallocAsync pool (miss); NULL on failure.  A 0-byte
 * request returns a valid handle with no storage.  Replaces shim.h:42-44. */
void* nxv_buf_alloc(unsigned long n_bytes);

/* Return a buffer to the pool (at most 64 per size class; beyond that the
 * memory is released).  NULL is ignored.  Replaces shim.h:46-49. */
void nxv_buf_free(void* handle);

/* Release every pooled buffer and trim the device pool.  Replaces shim.h:51-54. */
void nxv_pool_clear(void);

/* Pool counters; any pointer may be NULL.  Replaces shim.h:56-59. */
void nxv_pool_stats(unsigned long* hits, unsigned long* misses,
                    unsigned long* freed, unsigned long* size_classes,
                    unsigned long* total_pooled);

/* Copy n_bytes host->device (<= the buffer size).  Pinned host memory is
 * copied directly; pageable memory goes through a pinned staging ring.
 * Replaces shim.h:61-62. */
int nxv_buf_upload(void* handle, const void* data, unsigned long n_bytes);

/* Copy n_bytes device->host (<= the buffer size) and wait for it.
 * Replaces shim.h:64-65. */
int nxv_buf_download(void* handle, void* data, unsigned long n_bytes);

/* ---- Elementwise (shim.h:69-86, 122-127, 136-146) ---------------------- */

/* out = a op b over n elements.  op 0 add 1 mul 2 sub 3 div 4 pow 5 max
 * 6 min 7 equal 8 less 9 greater (comparisons give 1.0/0.0).
 * spv basename: elementwise_binary.spv (f32) | elementwise_binary_f64.spv.
 * Replaces shim.h:77-79. */
int nxv_apply_binary(void* out, void* a, void* b,
                     unsigned int n, unsigned int op,
                     const char* spv_path);

/* out = op(a).  op 0 exp 1 log 2 sqrt 3 abs 4 neg 5 sigmoid 6 tanh 7 relu
 * 8 ceil 9 floor 10 sign 11 reciprocal 12 square 13 erf 14 expm1.
 * spv: elementwise_unary.spv | elementwise_unary_f64.spv (true f64 math;
 * the reference evaluated f64 transcendentals through f32, backend.ex:309-311).
 * Replaces shim.h:84-86. */
int nxv_apply_unary(void* out, void* a,
                    unsigned int n, unsigned int op,
                    const char* spv_path);

/* spv: cast_f32_to_f64.spv | cast_f64_to_f32.spv.  Replaces shim.h:125-127. */
int nxv_cast(void* out, void* a,
             unsigned int n,
             const char* spv_path);

/* Strided broadcast binary, ndim 1..4, stride 0 broadcasts; out is dense
 * row-major over out_shape.  spv: elementwise_binary_broadcast.spv |
 * elementwise_binary_broadcast_f64.spv.  Replaces shim.h:141-146. */
int nxv_apply_binary_broadcast(void* out, void* a, void* b,
                               unsigned int op, unsigned int ndim,
                               const unsigned int* out_shape,
                               const unsigned int* a_strides,
                               const unsigned int* b_strides,
                               const char* spv_path);

/* 2-D transpose, C[j,i] = A[i,j], f32 (transpose.spv) or f64
 * (transpose_f64.spv).  Replaces shim.h:118-120. */
int nxv_transpose(void* out, void* a,
                  unsigned int m, unsigned int n,
                  const char* spv_path);

/* ---- Fused op tape (shim.h:148-167) ------------------------------------ */

/* r = a[i]; up to 8 ops left to right; binary 0..6 take b[i]; unary
 * 100..114; 255 = nop.  f32 (fused_elementwise.spv).  Replaces shim.h:155-158. */
int nxv_fused_chain(void* out, void* a, void* b,
                    unsigned int n, unsigned int n_ops,
                    const unsigned int* ops,
                    const char* spv_path);

/* As nxv_fused_chain with 4 inputs; buf_idx[k] in {1,2,3} picks b/c/d for
 * binary step k.  f32 (fused_elementwise_4in.spv).  Replaces shim.h:163-167. */
int nxv_fused_chain_4(void* out, void* a, void* b, void* c, void* d,
                      unsigned int n, unsigned int n_ops,
                      const unsigned int* ops,
                      const unsigned int* buf_idx,
                      const char* spv_path);

/* NEW.  Op tape with immediate scalars and a dtype: src[k] = 0 takes the
 * scalar imm[k] (rounded to the chain type) as the right operand of binary
 * step k, 1/2/3 take b/c/d; binary ops 0..9.  dtype 0 = f32, 1 = f64.
 * b/c/d may be NULL when no step reads them.  This is the lowering target
 * of the chain compiler for chains with literals such as
 * tanh(exp(x*y + z) - 1.0), which the reference cannot fuse
 * (lib/nx_vulkan/compiler.ex:291-307).  spv: fused_elementwise_imm.spv. */
int nxv_fused_chain_imm(void* out, void* a, void* b, void* c, void* d,
                        unsigned int n, unsigned int n_ops,
                        const unsigned int* ops,
                        const unsigned int* src,
                        const double* imm,
                        unsigned int dtype,
                        const char* spv_path);

/* ---- Reductions (shim.h:88-92, 129-134) -------------------------------- */

/* Full reduce of n f32 to a host scalar; op 0 sum 1 min 2 max.  Sums
 * accumulate in f64 and round once.  spv: reduce.spv.  Replaces shim.h:90-92. */
int nxv_reduce(float* out_scalar, void* in,
               unsigned int n, unsigned int op,
               const char* spv_path);

/* (outer, R, inner) -> (outer, inner); op 0 sum 1 max 2 min.
 * spv: reduce_axis.spv | reduce_axis_f64.spv | logsumexp.spv (f32; op
 * ignored).  Replaces shim.h:131-134 (and lib.rs:927-961 for logsumexp). */
int nxv_reduce_axis(void* out, void* a,
                    unsigned int outer, unsigned int reduce_size, unsigned int inner,
                    unsigned int op,
                    const char* spv_path);

/* NEW.  f64 full reduce to a host double; op 0 sum 1 min 2 max.  Sums use
 * double-double accumulation in a fixed order (deterministic).  Wires the
 * reference's unwired reduce_full_f64.spv (248_TODO.md:55-57).
 * spv: reduce_full_f64.spv. */
int nxv_reduce_f64(double* out_scalar, void* in,
                   unsigned long n, unsigned int op,
                   const char* spv_path);

/* NEW.  Full reduce into a 1-element device buffer of the input's type
 * (no host round trip; replaces backend.ex:459-463 scalar_to_tensor).
 * dtype 0 f32, 1 f64.  spv: reduce.spv | reduce_full_f64.spv. */
int nxv_reduce_to_buf(void* out, void* in,
                      unsigned long n, unsigned int op, unsigned int dtype,
                      const char* spv_path);

/* NEW.  argmax (is_min = 0) / argmin (1) over R of (outer, R, inner) into
 * (outer, inner) indices; lowest index on ties (Nx tie_break: :low); a NaN
 * beats every number and the first NaN wins.  dtype 0 f32, 1 f64;
 * index_bytes 4 (s32) or 8 (s64).  The reference computes this on the host
 * (lib/nx_vulkan/backend.ex:1188-1191).  spv: argmax_axis.spv. */
int nxv_argmax_axis(void* out, void* a,
                    unsigned int outer, unsigned int reduce_size, unsigned int inner,
                    unsigned int is_min, unsigned int dtype, unsigned int index_bytes,
                    const char* spv_path);

/* ---- Matmul (shim.h:94-109) -------------------------------------------- */

/* C[M,N] = A[M,K] . B[K,N], row-major.  f32 through 3xTF32 on the tcgen05
 * tensor cores.  Any of matmul*.spv selects it.  Replaces shim.h:95-97. */
int nxv_matmul(void* out, void* a, void* b,
               unsigned int m, unsigned int n, unsigned int k,
               const char* spv_path);

/* Same; tile_m/tile_n are accepted for ABI compatibility and ignored (the
 * kernel picks its own tiles).  Replaces shim.h:106-109. */
int nxv_matmul_v(void* out, void* a, void* b,
                 unsigned int m, unsigned int n, unsigned int k,
                 unsigned int tile_m, unsigned int tile_n,
                 const char* spv_path);

/* NEW.  Batched C[q] = A[q] . B[q] for q < batch (Nx.dot with batch axes
 * [0]/[0]); dtype 0 f32 (3xTF32), 1 f64 (DMMA tensor cores).  batch = 1 is
 * a plain f64 matmul (the reference sends f64 dot to the host,
 * backend.ex:480-485).  spv: matmul_batched.spv. */
int nxv_matmul_batched(void* out, void* a, void* b,
                       unsigned int batch, unsigned int m, unsigned int n,
                       unsigned int k, unsigned int dtype,
                       const char* spv_path);

/* ---- Random (shim.h:111-114) ------------------------------------------- */

/* n f32 values from counter-based Philox-2x32-10; dist 0 U[0,1), 1 N(0,1)
 * (Box-Muller).  Element i depends only on (seed, i).  random_philox.spv.
 * Replaces shim.h:113-114. */
int nxv_random(void* out, unsigned int n, unsigned int seed, unsigned int dist,
               const char* spv_path);

/* NEW.  Same generator, f64 output (53-bit uniforms).  random_philox_f64.spv. */
int nxv_random_f64(void* out, unsigned long n, unsigned int seed, unsigned int dist,
                   const char* spv_path);

/* ---- Fused HMC primitives (shim.h:169-189) ----------------------------- */

/* Partial sums 0.5*sum(p^2*inv_mass), one f32 per 256-element group
 * (out has ceil(n/256) floats).  Replaces shim.h:171-173. */
int nxv_kinetic_energy(void* out, void* p, void* inv_mass,
                       unsigned int n,
                       const char* spv_path);

/* -0.5*((x-mu)/sigma)^2 - log(sigma) - 0.5*log(2 pi).  Replaces shim.h:177-179. */
int nxv_normal_logpdf(void* out, void* x, void* mu, void* sigma,
                      unsigned int n,
                      const char* spv_path);

/* One leapfrog step, Normal(mu, sigma).  Replaces shim.h:185-189. */
int nxv_leapfrog_normal(void* q_new, void* p_new,
                        void* q, void* p, void* inv_mass,
                        unsigned int n,
                        float eps, float mu, float sigma,
                        const char* spv_path);

/* ---- Fused K-step leapfrog chains (shim.h:191-280) ----------------------
 * Per step k: p_h = p + eps/2*grad(q); q = q + eps*inv_mass*p_h;
 * p = p_h + eps/2*grad(q) (the corrected sign, PLAN_FUSED_LEAPFROG.md:18-24).
 * q/p/grad chains are [k][i] (K*n elements); logp is [k].  The reference
 * limits these to n <= 256 (one workgroup); this library accepts any n. */

int nxv_leapfrog_chain_normal(void* q_chain, void* p_chain,
                              void* grad_chain, void* logp_chain,
                              void* q_init, void* p_init, void* inv_mass,
                              unsigned int n, unsigned int K,
                              float eps, float mu, float sigma,
                              const char* spv_path);               /* shim.h:197-202 */

/* partial_logp is [k][w] for w < num_workgroups = ceil(n/256): the sum over
 * elements 256w..256w+255 of step k; partial 0 carries the constant. */
int nxv_leapfrog_chain_normal_lg(void* q_chain, void* p_chain,
                                 void* grad_chain, void* partial_logp,
                                 void* q_init, void* p_init, void* inv_mass,
                                 unsigned int n, unsigned int K,
                                 unsigned int num_workgroups,
                                 float eps, float mu, float sigma,
                                 const char* spv_path);            /* shim.h:210-216 */

int nxv_leapfrog_chain_exponential(void* q_chain, void* p_chain,
                                   void* grad_chain, void* logp_chain,
                                   void* q_init, void* p_init, void* inv_mass,
                                   unsigned int n, unsigned int K,
                                   float eps, float lambda,
                                   const char* spv_path);          /* shim.h:222-227 */

int nxv_leapfrog_chain_studentt(void* q_chain, void* p_chain,
                                void* grad_chain, void* logp_chain,
                                void* q_init, void* p_init, void* inv_mass,
                                unsigned int n, unsigned int K,
                                float eps, float mu, float sigma,
                                float nu, float logp_const,
                                const char* spv_path);             /* shim.h:231-237 */

int nxv_leapfrog_chain_cauchy(void* q_chain, void* p_chain,
                              void* grad_chain, void* logp_chain,
                              void* q_init, void* p_init, void* inv_mass,
                              unsigned int n, unsigned int K,
                              float eps, float loc, float scale,
                              float log_pi_scale,
                              const char* spv_path);               /* shim.h:241-247 */

int nxv_leapfrog_chain_halfnormal(void* q_chain, void* p_chain,
                                  void* grad_chain, void* logp_chain,
                                  void* q_init, void* p_init, void* inv_mass,
                                  unsigned int n, unsigned int K,
                                  float eps, float sigma, float log_const,
                                  const char* spv_path);           /* shim.h:252-257 */

int nxv_leapfrog_chain_weibull(void* q_chain, void* p_chain,
                               void* grad_chain, void* logp_chain,
                               void* q_init, void* p_init, void* inv_mass,
                               unsigned int n, unsigned int K,
                               float eps, float k, float lambda,
                               float logp_const,
                               const char* spv_path);              /* shim.h:264-270 */

int nxv_leapfrog_chain_normal_f64(void* q_chain, void* p_chain,
                                  void* grad_chain, void* logp_chain,
                                  void* q_init, void* p_init, void* inv_mass,
                                  unsigned int n, unsigned int K,
                                  double eps, double mu, double sigma,
                                  const char* spv_path);           /* shim.h:275-280 */

/* NEW.  Batched f64 Gaussian chains: n_chains independent chains, one launch.
 * grad = -prec .* (q - mu); logp = -0.5 sum prec (q-mu)^2 + 0.5 sum log prec
 * - n/2 log 2pi.  q_init, p_init are [chain][i]; inv_mass is [chain][i],
 * or one [i] row used by every chain when its buffer holds exactly n
 * doubles and n_chains > 1 (Nx broadcasting of an [i] mass over the chains,
 * lib/nx_vulkan.ex:808-835; the [i] form uploads n instead of n_chains * n
 * doubles); prec is [i] (shared); q/p/grad chains are [chain][k][i]; logp is
 * [chain][k].  With n_chains = 1 and prec = 1/sigma^2 this is
 * nxv_leapfrog_chain_normal_f64.
 * spv: leapfrog_chain_gauss_f64_batched.spv. */
int nxv_leapfrog_chain_gauss_f64_batched(void* q_chain, void* p_chain,
                                         void* grad_chain, void* logp_chain,
                                         void* q_init, void* p_init, void* inv_mass,
                                         void* prec,
                                         unsigned int n, unsigned int n_chains,
                                         unsigned int K, double eps, double mu,
                                         const char* spv_path);

/* NEW.  nxv_leapfrog_chain_gauss_f64_batched that also writes the kinetic
 * energy of every step, ke_chain[chain][k] = 0.5 * sum_i p_i^2 * inv_mass_i
 * (the reference's kinetic_energy.spv formula, shim.h:169-173, fused into
 * the chain's epilogue so a NUTS caller gets the Hamiltonian -logp + KE of
 * every trajectory point without another pass).  ke_chain holds
 * n_chains * K doubles; inv_mass may be [i] as above.
 * spv: leapfrog_chain_gauss_f64_batched.spv. */
int nxv_leapfrog_chain_gauss_f64_batched_ke(void* q_chain, void* p_chain,
                                            void* grad_chain, void* logp_chain,
                                            void* ke_chain,
                                            void* q_init, void* p_init, void* inv_mass,
                                            void* prec,
                                            unsigned int n, unsigned int n_chains,
                                            unsigned int K, double eps, double mu,
                                            const char* spv_path);

/* NEW, with no counterpart in the reference.  The batched f64 Gaussian
 * chain above for callers that must not allocate device memory while they
 * run: a framework that reserves GPU memory for its own allocator and hands
 * its kernels raw device buffers (XLA/EXLA preallocate most of HBM, so a
 * side allocation by this library can fail), or a service that does all of
 * its device allocation at start-up and keeps a fixed memory budget.
 * Arguments are raw device pointers, not nxv handles, laid out as in
 * nxv_leapfrog_chain_gauss_f64_batched; the caller guarantees their sizes.
 * The call allocates nothing: its scratch is a 1 MiB static device array
 * that every GPU loading this library holds until the process exits.
 * Limit: chains of n <= 2048 elements need only 256 bytes of it; longer
 * chains also need n_chains * K * ceil(n / 2048) partial sums of 8 bytes
 * (2048 is the default kernel's tile; the NXV_LF_TMA and NXV_LF_CFG tuning
 * variables can change it), and a call needing more than 1 MiB returns -3
 * with a message naming the limit.  nxv_init (or nxv_init_devices) must have run.  The first call on
 * a device looks up the array's device address and must come before any
 * stream capture.  All calls share the array: two calls that overlap on
 * the GPU (different streams or threads) race.  Nothing in it needs
 * clearing between calls.  Same results as the allocating entry point. */
int nxv_leapfrog_chain_gauss_f64_batched_noalloc(void* q_chain, void* p_chain,
                                                 void* grad_chain, void* logp_chain,
                                                 const void* q_init, const void* p_init,
                                                 const void* inv_mass, const void* prec,
                                                 unsigned int n, unsigned int n_chains,
                                                 unsigned int K, double eps, double mu);

/* NEW.  Batched f64 Bayesian logistic-regression chains (inv_mass = 1):
 * grad(q) = X^T (y - sigmoid(X q)) - q,
 * logp(q) = sum_j [y_j z_j - log(1 + e^{z_j})] - 0.5 |q|^2, z = X q.
 * X is [n_obs][n_dim], y is [n_obs] (0/1 as f64), q_init/p_init are
 * [chain][n_dim]; outputs as in the Gaussian batch.  The gradient is two
 * f64 GEMMs per step on the DMMA tensor cores.
 * spv: leapfrog_logreg_f64_batched.spv. */
int nxv_leapfrog_logreg_f64_batched(void* q_chain, void* p_chain,
                                    void* grad_chain, void* logp_chain,
                                    void* q_init, void* p_init,
                                    void* X, void* y,
                                    unsigned int n_obs, unsigned int n_dim,
                                    unsigned int n_chains, unsigned int K,
                                    double eps,
                                    const char* spv_path);

/* ---- NUTS tree builder on the device (NEW) ------------------------------
 * eXMC's NUTS tree builder (an external repository; its call site is
 * PLAN_FUSED_LEAPFROG.md:331-358) walks the leaves that the fused chain
 * returns.  These calls do that walk on the device, over a leaf store
 * that the batched Gaussian chain (_ke variant) writes into, so the
 * trajectories never leave the GPU; the caller keeps the row bookkeeping
 * and draws the random numbers.  Store rows hold q, p (p in its
 * integration sign: negated for backward leaves), logp and the kinetic
 * energy; H = -logp + KE.  Arrays of chain / slot indices and directions
 * are int32, store rows int64, the rest f64.  0 on success, -1 NULL, -3 a
 * buffer smaller than its extent. */

/* H0[c] = 0.5 sum prec (q - mu)^2 - logp_const + 0.5 sum p^2 inv_mass over
 * [n_chains][d] q and p (the Gaussian target's Hamiltonian). */
int nxv_nuts_energy(void* H0, void* q, void* p, void* prec, void* inv_mass,
                    double mu, double logp_const,
                    unsigned int n_chains, unsigned int d);

/* Starting points of a speculative extension of chains chain[i] (i < n_need):
 * store row src_row[i], or the initial point (q0[c], dir[i] * p0[c]) when
 * src_row[i] < 0; written to qs, ps [n_need][d]. */
int nxv_nuts_start(void* qs, void* ps, void* q0, void* p0, void* st_q, void* st_p,
                   void* chain, void* src_row, void* dir,
                   unsigned int n_need, unsigned int n_chains, unsigned int d);

/* One tree level for n_active chains: slot a is chain chain[a], whose new
 * subtree is the n (a power of two, <= 2048) store rows rows[a][0..n) in time
 * order, extending the tree forward (fwd[a] = 1) or backward.  Per chain:
 * divergence (H - H0 > 1000 or NaN), the subtree's U-turn checks, the
 * multinomial leaf (u_sel[a]) and the biased move (u_move[a]) into `sample`,
 * logw, the merge checks with the tree (rho, end_p / end_ps: [2][C][d], left
 * end first), active[c] (1 while the tree grows) and divergent[c].  node:
 * [n_active][n][d] f64 scratch. */
int nxv_nuts_level(void* rows, void* chain, void* fwd, void* u_sel, void* u_move,
                   unsigned int n_active, unsigned int n, unsigned int d,
                   void* st_q, void* st_p, void* st_logp, void* st_ke, void* inv_mass,
                   void* H0, void* logw, void* rho, void* end_p, void* end_ps,
                   void* sample, void* active, void* divergent, void* node,
                   unsigned int n_chains);

/* Device-driven levels: the tree's state stays on the device and every
 * chain's level-l leaves sit at fixed store rows base_row + c n + i
 * (i < n = 2^l, in integration order; base_row = n_chains (2^l - 1) when the
 * levels are stacked), so that a driver launches one start, one chain call
 * into those rows and one level call per level without reading anything
 * back but the active flags.  u: [3][n_chains] uniforms of the level --
 * direction (forward when >= 0.5), leaf, move.  end_row: [2][n_chains]
 * int64 store row of each tree's left / right end leaf, -1 for the initial
 * point. */

/* Starting points of level u_dir's extension for every chain: the end
 * leaf on the chosen side, or (q0[c], +-p0[c]) while that side has none;
 * written to qs, ps [n_chains][d]. */
int nxv_nuts_start_layout(void* qs, void* ps, void* q0, void* p0, void* st_q, void* st_p,
                          void* end_row, void* u_dir, unsigned int n_chains,
                          unsigned int d);

/* One level for every chain still building (active[c] = 1): the walk of
 * nxv_nuts_level over rows base_row + c n .. + n - 1 (reversed in time for a
 * backward extension), then end_row of that side, depth[c] = level + 1 and
 * n_leapfrog[c] += n (int32).  node: [n_chains][n][d] f64 scratch.  -3 also
 * when the store holds fewer than base_row + n_chains n rows. */
int nxv_nuts_level_layout(unsigned long long base_row, unsigned int n, unsigned int d,
                          void* u, void* st_q, void* st_p, void* st_logp, void* st_ke,
                          void* inv_mass, void* H0, void* logw, void* rho, void* end_p,
                          void* end_ps, void* sample, void* active, void* divergent,
                          void* end_row, void* depth, void* n_leapfrog, void* node,
                          unsigned int n_chains, unsigned int level);

/* One whole NUTS transition of every chain in one call, with the levels
 * above run by the library: momenta p0 = N(0, 1) / sqrt(inv_mass) and the
 * per-level uniforms [max_depth][3][n_chains] drawn by Philox-2x32-10 (the
 * nxv_random_f64 streams of keys seed and seed ^ 0x5BD1E995), the initial
 * energy, then per level one start kernel, one batched Gaussian chain call
 * of 2^l steps (with kinetic energy) into the library's own leaf store and
 * one level kernel, with one 4-byte read per level (from the third on) of
 * whether any tree still grows.  q0 [n_chains][d], inv_mass and prec [d] (the Gaussian
 * target's diagonal precision and mean mu, logp_const the log density's
 * constant); outputs sample [n_chains][d], flags [4][n_chains] int32
 * (active at the end, divergent, depth, leapfrog steps) and H0 [n_chains]
 * (initial energy).  The tree state and the store (n_chains (2^max_depth -
 * 1) leaves) live in library scratch, kept for the next call.  -3 when
 * max_depth is outside 1..12.  The level kernels run on a second stream of
 * the library, ordered with the caller's stream by events, so that each
 * level's walk overlaps the next level's chain call.  Returns after the
 * last level's flag read (the call synchronises with the device once per
 * level, so it cannot be captured into a CUDA graph); the outputs are
 * complete in the caller's stream order. */
int nxv_nuts_transition_layout(void* sample, void* flags, void* H0, void* q0, void* inv_mass,
                               void* prec, double mu, double logp_const, double eps,
                               unsigned int n_chains, unsigned int d, unsigned int max_depth,
                               unsigned int seed);

/* ---- Devices, streams, interop (NEW) ----------------------------------- */

/* Use exactly these CUDA devices (e.g. the local rank's GPU).  Calls nxv_init
 * semantics for each; device ids[0] becomes current.  0 on success. */
int nxv_init_devices(const int* ids, int n);

/* Make device `id` (one of the initialised ones) current for the calling
 * thread.  Buffers remember their device; an op on buffers of another
 * device returns -3. */
int nxv_set_device(int id);

/* Run this thread's work for the current device on a caller-owned
 * cudaStream_t (passed as void*); NULL restores the library's own stream.
 * To use the legacy default stream pass cudaStreamLegacy ((void*)1). */
int nxv_set_stream(void* cuda_stream);

/* Wait for all work queued on the current device.  0, or -4 with the CUDA
 * error that a kernel raised. */
int nxv_synchronize(void);

/* Non-owning handle over existing device memory of n_bytes (e.g. a tensor
 * of another framework); nxv_buf_free releases only the handle record.  The
 * caller keeps that memory allocated for as long as work using the handle
 * can run -- including CUDA graphs captured with it, which keep its raw
 * address. */
void* nxv_buf_wrap(void* device_ptr, unsigned long n_bytes);

/* NEW.  Device-to-device copy of `rows` rows of `width` bytes: row r is read
 * at byte src_offset + r * src_pitch of src and written at dst_offset +
 * r * dst_pitch of dst (one cudaMemcpy2DAsync on the current stream, no
 * kernel).  A strided slice of a device tensor without a host round trip,
 * e.g. the last step q_chain[:, K-1, :] of a batched chain as the next
 * trajectory's q_init.  The reference's Backend.slice downloads the tensor,
 * walks the output coordinates on the host and uploads the result
 * (lib/nx_vulkan/backend.ex:665-720); this is the device form of its
 * contiguous-row case.  0 on success, -1 for a NULL handle, -3 when a row
 * would leave a buffer. */
int nxv_buf_copy_2d(void* dst, unsigned long dst_offset, unsigned long dst_pitch,
                    void* src, unsigned long src_offset, unsigned long src_pitch,
                    unsigned long width, unsigned long rows);

/* Device address and byte size behind a handle (NULL / 0 for NULL). */
void* nxv_buf_device_ptr(void* handle);
unsigned long nxv_buf_size(void* handle);

/* Last error message of the calling thread ("" when none). */
const char* nxv_last_error(void);

/* Number of this library's kernel launches since load (all threads). */
unsigned long nxv_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif
