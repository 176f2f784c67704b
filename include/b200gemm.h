/*
 * b200gemm: bf16 x bf16 -> bf16 GEMM (fp32 accumulate) for NVIDIA B200
 * (sm_100a), C = A . B^T with
 *   A: M x K, row-major (K contiguous, leading dimension K)
 *   B: N x K, row-major (K contiguous, leading dimension K)
 *   C: M x N, row-major, leading dimension ldc >= N
 * Output elements are the fp32 sums rounded to bf16 (round to nearest even).
 *
 * This header is the drop-in boundary for the reference project's launcher
 *   void runKernel1(int M, int N, int K, bf16 *A, bf16 *B, bf16 *C, int *DB)
 *   (b200_kernels/matmul_1.cuh:386-418, exported at :422, dispatched from
 *    run_kernel() in matmul_b200.cu:28-38).
 * Differences from that launcher, all in the caller's favour: explicit
 * stream, status codes instead of exit(1) (reference include/utils.cuh:13-20),
 * a per-handle descriptor cache keyed on every argument (the reference keys
 * its cache on M only, matmul_1.cuh:390), any M, N >= 0 and K % 8 == 0
 * (the reference needs K % 64 == 0 and full 256 x 256 tiles).
 *
 * All entry points are thread-safe per handle.  Plain C types only.
 */
#ifndef B200GEMM_H_
#define B200GEMM_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define B200GEMM_OK 0
#define B200GEMM_ERR_INVALID_ARG 1   /* null handle/pointer, negative size      */
#define B200GEMM_ERR_UNSUPPORTED 2   /* K % 8, ldc % 8, ldc < N, misaligned ptr  */
#define B200GEMM_ERR_CUDA 3          /* a CUDA runtime/driver call failed        */
#define B200GEMM_ERR_DEVICE_TIMEOUT 4 /* a bounded wait inside a kernel ran out   */
#define B200GEMM_ERR_NO_DEVICE 5     /* device missing or not sm_100             */
#define B200GEMM_ERR_TOO_LARGE 6     /* a dimension exceeds the supported range  */

typedef struct b200gemm_handle* b200gemm_t;

/* Create a handle bound to CUDA device `device`.  Allocates a few bytes of
 * device memory for the status words.  Replaces the reference's hidden
 * globals d_tma_map_A/B/C, _prev_m/n/k and _dspace (matmul_1.cuh:5-11). */
int b200gemm_create(b200gemm_t* handle, int device);

/* Release the handle and every device buffer it owns. */
void b200gemm_destroy(b200gemm_t handle);

/* C = A . B^T (see top of file).  Asynchronous on `stream` (a cudaStream_t,
 * NULL = legacy default stream).  A, B, C must be 16-byte aligned device
 * pointers on the handle's device; K % 8 == 0; ldc % 8 == 0; ldc >= N.
 * The first call for a new (M, N) tile grid builds the tile schedule and
 * waits for it (one-time, per handle).
 * Replaces runKernel1 (matmul_1.cuh:386-418). */
int b200gemm_bf16_nt(b200gemm_t handle, int M, int N, int K, const void* A, const void* B,
                     void* C, int ldc, void* stream);

/* Fused epilogue, applied per element in fp32 to the accumulator before C is
 * written (the ops around an MLP projection, without a second pass over C):
 *     D[i][j] = act(alpha * (A . B^T)[i][j] + bias[j]) + beta * residual[i][j]
 * then C[i][j] = D[i][j] rounded to bf16 (RNE), stored as fp32, or scaled by
 * out_scale and rounded to fp8 e4m3 (OCP FP8 E4M3: RNE, saturating to
 * +-448).  A NULL bias or residual drops that term.  No counterpart in the reference, whose
 * epilogue only rounds the accumulator to bf16 (matmul_1.cuh:293-295). */
#define B200GEMM_ACT_NONE 0
#define B200GEMM_ACT_RELU 1       /* max(x, 0)                                   */
#define B200GEMM_ACT_GELU 2       /* 0.5 x (1 + erf(x / sqrt 2))                 */
#define B200GEMM_ACT_GELU_TANH 3  /* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) */
#define B200GEMM_ACT_SILU 4       /* x / (1 + exp(-x))                           */
#define B200GEMM_OUT_BF16 0
#define B200GEMM_OUT_F32 1
#define B200GEMM_OUT_E4M3 2
typedef struct b200gemm_epilogue {
  float alpha;           /* scale of A . B^T                                     */
  float beta;            /* scale of the residual                                */
  const void* bias;      /* bf16[N] device vector, 16-byte aligned, or NULL      */
  const void* residual;  /* bf16 M x N device matrix, row pitch ldr, or NULL     */
  int ldr;               /* residual pitch in elements: ldr >= N, ldr % 8 == 0,  */
                         /* residual 16-byte aligned                             */
  int activation;        /* B200GEMM_ACT_*                                       */
  int out_type;          /* B200GEMM_OUT_BF16, B200GEMM_OUT_F32 (C holds fp32,   */
                         /* ldc in fp32 elements, ldc % 4 == 0) or               */
                         /* B200GEMM_OUT_E4M3 (C holds bytes, ldc % 16 == 0)     */
  float out_scale;       /* e4m3 output: C = e4m3(out_scale * D); 0 means 1      */
} b200gemm_epilogue;

/* C = epilogue(A . B^T) with the epilogue above; epi == NULL is exactly
 * b200gemm_bf16_nt.  Same rules as b200gemm_bf16_nt, plus K > 0 and those in
 * the struct.  Runs the kernel b200gemm_bf16_nt would run for the shape (the
 * small-M kernels where it would, except e4m3 output with N % 16 != 0); the
 * tiled kernel's width accounts for the epilogue's cost (a costly epilogue
 * favours 256-wide tiles, whose epilogue overlaps the next tile's MMAs).
 * Every tile width sums an element's K products in the same order, so the
 * accumulator is bit-identical to b200gemm_bf16_nt's. */
int b200gemm_bf16_nt_epilogue(b200gemm_t handle, int M, int N, int K, const void* A,
                              const void* B, void* C, int ldc, const b200gemm_epilogue* epi,
                              void* stream);

/* C = A . B^T with A, B and C in host memory (pinned memory lets the copies
 * overlap; pageable memory works but serialises).  The handle stages the
 * operands in device buffers it owns (allocated on first use, grown when
 * needed): B is copied first, then A and C move in (about 3) row chunks of
 * whole 256-row tiles on separate streams, so the copy of chunk i+1, the GEMM of
 * chunk i and the copy-out of chunk i-1 overlap.  Asynchronous with respect
 * to the host: completion is ordered on `stream`, and the host buffers must
 * stay valid until then.  Consecutive calls alternate between two sets of
 * device buffers, so a call on another stream uploads its operands while the
 * previous call's last GEMM and copy-out still run (a call on the same stream
 * starts after the previous one completes, as stream order requires).  Calls
 * on one handle are enqueued one at a time.  ldc is the
 * host row pitch of C (>= N); K % 8 == 0.  No reference counterpart (the
 * reference bench copies synchronously, matmul_b200.cu:80-83, 107-110). */
int b200gemm_bf16_nt_host(b200gemm_t handle, int M, int N, int K, const void* A, const void* B,
                          void* C, int ldc, void* stream);

/* GEMM with a fused all-gather of C for an N-sharded multi-GPU job (one
 * process per GPU, each computing its own block of columns of C).  The call
 * computes this rank's block into C like b200gemm_bf16_nt (C and ldc point at
 * the block's place inside this rank's full-width C), and the epilogue also
 * writes every finished 32 x 32 chunk straight into the same place of each
 * peer's full-width C over NVLink (peer_C[i]: this rank's block inside peer
 * i's C, same ldc; device pointers from b200gemm_ipc_open), so the gather
 * overlaps the GEMM instead of following it.  npeers <= 7; N % 8 == 0;
 * K > 0 (with K == 0 the peers' blocks would not be written).  When
 * `stream` completes the local and peer writes are done; the peers still
 * need a barrier with this rank before reading.  Always uses the tiled
 * kernel.  No reference counterpart (the reference has no multi-GPU code). */
int b200gemm_bf16_nt_allgather(b200gemm_t handle, int M, int N, int K, const void* A,
                               const void* B, void* C, int ldc, void* const* peer_C, int npeers,
                               void* stream);

/* The same fused all-gather through an NVLink multicast (NVLS) mapping of
 * every rank's full-width C: the epilogue writes each finished chunk once,
 * with multimem.st, to mc_C (the multicast address of this rank's block,
 * same ldc), and NVSwitch replicates it into every rank's C, this rank's
 * own included (the local copy is not written separately; C is only
 * described).  A multicast object spanning the ranks' C buffers comes from
 * the caller, e.g. torch's symmetric memory (shard.MulticastAllGather).
 * N % 8 == 0, K > 0, mc_C 16-byte aligned.  Every rank must keep its buffer
 * bound until all ranks are done with it: tear down collectively.  No
 * reference counterpart. */
int b200gemm_bf16_nt_allgather_multicast(b200gemm_t handle, int M, int N, int K, const void* A,
                                         const void* B, void* C, int ldc, void* mc_C, void* stream);

/* CUDA IPC helpers for sharing device buffers between the processes of a
 * multi-GPU job: export a handle (B200GEMM_IPC_HANDLE_BYTES bytes) for the
 * allocation holding dev_ptr plus dev_ptr's byte offset inside it, map a
 * peer's handle (returns the allocation base; add the offset; peer access is
 * enabled on first use), and unmap it. */
#define B200GEMM_IPC_HANDLE_BYTES 64
int b200gemm_ipc_get_handle(const void* dev_ptr, void* handle_out, unsigned long long* offset_out);
int b200gemm_ipc_open(const void* handle, void** dev_ptr_out);
int b200gemm_ipc_close(void* dev_ptr);

/* Waits for the handle's device, returns the first device-side error the
 * kernels recorded since the last call (B200GEMM_OK or
 * B200GEMM_ERR_DEVICE_TIMEOUT) and clears it.  `detail`, if non-null,
 * receives 4 words: code, site, CTA id, tile index.
 * No reference counterpart (its waits spin forever, b200_utils.cuh:451-463). */
int b200gemm_last_device_status(b200gemm_t handle, unsigned int* detail);

/* Budget for every bounded wait inside the kernels, in nanoseconds
 * (default 2e9).  No reference counterpart. */
int b200gemm_set_timeout_ns(b200gemm_t handle, unsigned long long timeout_ns);

/* Launch a two-CTA kernel whose only wait can never be satisfied, with the
 * given budget; afterwards b200gemm_last_device_status() must report
 * B200GEMM_ERR_DEVICE_TIMEOUT.  Exercises the watchdog without a fault.
 * No reference counterpart. */
int b200gemm_selftest_watchdog(b200gemm_t handle, unsigned long long timeout_ns, void* stream);

/* Drop-in for the reference launcher signature (matmul_1.cuh:386): uses a
 * process-wide handle for the current device, the legacy default stream and
 * ldc = N.  `DB` (the reference's debug buffer, unused by its B200 path,
 * matmul_b200.cu:35) is accepted and ignored. */
int b200gemm_run_kernel(int M, int N, int K, const void* A, const void* B, void* C, int* DB);

/* Launch geometry chosen for the handle's device: SM count and the number of
 * 2-CTA clusters of the GEMM kernel that fit on the device at once (the
 * persistent grid size).  Either pointer may be null.  The reference fixes
 * both at compile time (NUM_SM = 148, matmul_1.cuh:19). */
int b200gemm_device_info(b200gemm_t handle, int* sm_count, int* max_clusters);

/* Output tile width of the handle's GEMM calls: 256 (256 x 256 tiles, two
 * TMEM accumulators so a tile's epilogue overlaps the next tile's MMAs), 512
 * (256 x 512 tiles: one A stage feeds two MMAs, a quarter less operand
 * traffic per flop), 448 (the same with two N = 224 MMAs, so a shared-A tile
 * divides N = 1792 = 4 x 448), 224, 192 or 128 (narrower 256-row tiles, for
 * N that wider tiles split into a partly idle last wave), or 0 (default) to
 * choose per call from the shape.  Any other value is
 * B200GEMM_ERR_INVALID_ARG.  The reference has one fixed 256 x 256
 * configuration (matmul_1.cuh:13-22). */
int b200gemm_set_tile_width(b200gemm_t handle, int width);

/* Split the last, partial wave of tiles along K (default off): when T tiles
 * leave the last wave of G clusters partly idle, each of its T mod G tiles is
 * cut into up to 6 K slices run on the idle clusters (with T < G the single
 * wave is all tail and every tile is split); the slices write fp32
 * partials to a workspace owned by the handle and the last one to finish
 * adds them and writes C.  Split launches on one handle are serialised with
 * an event (they share the workspace).  No reference counterpart. */
int b200gemm_set_tail_split(b200gemm_t handle, int enable);

/* Run a short last wave of 256 x 512 (256 x 448) tiles as 256-column
 * (224-column) halves (default
 * on): when T tiles leave R = T mod G of G clusters busy in the last wave and
 * 2R <= G, each of those R tiles runs as two half tiles over the whole of K on
 * 2R clusters, so that wave takes about half a tile's time.  Plain epilogue
 * only.  No reference counterpart (its tiles are always 256 x 256). */
int b200gemm_set_tail_half(b200gemm_t handle, int enable);

/* Launch plan a call with this shape would use now, in plan[0..5]: kernel
 * (1 tiled, 2 small-M with 256 rows of B per CTA pair, 3 small-M with 128
 * rows of B per CTA), tile width (tiled) or rows of B per cluster (small-M),
 * tiles, clusters launched, how the tiles of the last partial wave are cut
 * (tiled kernel: 1 = not at all, S >= 2 = into S K slices, -2 = into two
 * half-width tiles), K split of the small-M kernel. */
int b200gemm_plan(b200gemm_t handle, int M, int N, int K, int* plan);

/* The tile width (512, 448, 256, 224, 192 or 128) a call with this shape would
 * use now; 0 for an invalid handle or shape. */
int b200gemm_tile_width_for(b200gemm_t handle, int M, int N, int K);

/* Small-M kernels (M <= 256, N % 8 == 0, K >= 128): rows of B become the
 * MMA's M side and K is split over 1, 2 or 4 CTA pairs of one cluster whose
 * fp32 partial sums are reduced through distributed shared memory, so every
 * SM streams B from HBM.  The CTA-pair form covers up to 256 rows of A, the
 * single-CTA form up to 128.  The CTA-pair form also runs small shapes of
 * 257..4096 rows of A (N % 8 == 0, K >= 256 split over 2 or 4 pairs) over
 * blocks of 128 or 256 rows of A, one cluster per block of B and A rows,
 * where all clusters fit at once and each CTA then loads fewer bytes than a
 * CTA of the tiled kernel would; never while a tile width is forced.
 * mode -1 (default) or 1: use them for eligible shapes; 0: always use the
 * tiled kernel.  The reference has no small-M path. */
int b200gemm_set_small_m(b200gemm_t handle, int mode);

/* Launch overlap with the previous kernel (programmatic dependent launch).
 * OFF (default): a call starts after the previous work on the stream.
 * ON: the kernel may be scheduled while the previous kernel on the stream is
 *   still running; it sets up (barriers, tensor memory) and then waits for
 *   that kernel to complete before any access to global memory, and it lets
 *   the next kernel launched this way start its own setup while it finishes.
 * WEIGHTS_EARLY: as ON, and the first ring of B (the weights) is requested
 *   before that wait, so streaming B overlaps the previous kernel's tail.
 *   The caller guarantees that the previous kernel does not write B.
 * The tiled kernel takes WEIGHTS_EARLY as ON: it reads its tile
 * table before any operand.  The multi-GPU all-gather form never overlaps.
 * Work on the stream other than these kernels (copies, events, other
 * kernels) keeps plain stream order.  The reference launches one kernel per
 * call with no overlap (matmul_1.cuh:416). */
#define B200GEMM_PDL_OFF 0
#define B200GEMM_PDL_ON 1
#define B200GEMM_PDL_WEIGHTS_EARLY 2
int b200gemm_set_pdl(b200gemm_t handle, int mode);

/* The K split (1, 2 or 4) the small-M kernel (pair or single-CTA form, see
 * b200gemm_plan) would use for this shape on this handle, or 0 when the
 * tiled kernel would run. */
int b200gemm_small_m_split(b200gemm_t handle, int M, int N, int K);

/* Tile orders for the persistent schedule. */
#define B200GEMM_ORDER_HILBERT 0 /* Hilbert curve over the tile grid           */
#define B200GEMM_ORDER_BANDS 1   /* bands of `band` tile-rows, columns swept    */

/* Select the order in which the handle's kernels start their 256 x 256
 * output tiles (entry j of the order runs on cluster j mod clusters).
 * Applies to calls made after it.  Replaces the fixed Hilbert table of the
 * reference (createHilbert, include/hilbert.hpp:42-84). */
int b200gemm_set_schedule(b200gemm_t handle, int order, int band);

/* Host computation of the schedule for a tiles_m x tiles_n grid of
 * 256 x 256 output tiles: out[0 .. tiles_m*tiles_n) receives
 * (tile_m << 16 | tile_n) in start order.  The device builds the identical
 * table.  Replaces createHilbert (include/hilbert.hpp:42-84).  Needs no GPU. */
int b200gemm_schedule_host(unsigned int tiles_m, unsigned int tiles_n, int order, int band,
                           unsigned int* out);

/* C = A . B^T like b200gemm_bf16_nt (same layouts, alignment and K/ldc
 * rules, asynchronous on `stream`, current device), for callers that must
 * not allocate device memory on the GEMM path: a memory pool or caching
 * allocator that runs GEMMs inside its own bookkeeping, a server that plans
 * all device memory up front and may not allocate later (an allocation can
 * block on the device or fail under fragmentation), or code that cannot
 * keep a handle.  It takes no handle and calls no cudaMalloc/cudaFree or
 * other allocating routine; its scratch (status words and the tile schedule)
 * is one static array of 64 KB + 256 B inside this library, which every GPU
 * that loads the library keeps until exit.
 *  - Limit: the output may need at most 16384 tiles (256 x 256 or 256 x 512,
 *    chosen per shape; e.g. 32768 x 32768 fits); larger problems return
 *    B200GEMM_ERR_TOO_LARGE before any GPU work.
 *  - The first call on a device sets up that device (looks up the array's
 *    device address, sets kernel attributes, loads every kernel this entry
 *    point launches); make it before any stream capture.
 *  - All calls share the array, which keeps the last call's contents; each
 *    call clears the status words and rewrites the schedule on `stream`, so
 *    calls that overlap on the GPU (different streams, not ordered) race.
 *  - Device-side watchdog timeouts are recorded in the array only; they are
 *    not reported through this call.
 * No counterpart in the reference. */
int b200gemm_bf16_nt_noalloc(int M, int N, int K, const void* A, const void* B, void* C, int ldc,
                             void* stream);

/* Human-readable text for a status code (static storage). */
const char* b200gemm_strerror(int code);

/* Library version as 10000*major + 100*minor + patch. */
int b200gemm_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* B200GEMM_H_ */
