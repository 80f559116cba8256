/*
 * semx.h — C ABI of the B200 (sm_100a) recurrent-scan library `libsemx.so`.
 *
 * The library implements the recurrent scans that sit inside the TF-blocks of the
 * SEMamba generator of a-baur/SEMambaXLinOSS:
 *   - the LinOSS oscillatory scan (IM / IMEX / damped IMEX, and the generic 2x2 form),
 *   - the selective-LRU diagonal scan (SISO, real and complex),
 *   - the selective-LRU MIMO scan with its block-diagonal readout,
 *   - the plain complex diagonal scan.
 * Each op has a forward and a backward entry point.
 *
 * Conventions (every entry point):
 *   - All pointers are device pointers to fp32 data (complex tensors are interleaved
 *     (re, im) pairs, i.e. the memory of a torch complex64 tensor), C-contiguous in the
 *     documented shape.
 *   - The first field of every argument struct is `struct_size`, which the caller sets to
 *     sizeof(struct); a mismatch returns SEMX_ERR_ABI.
 *   - Work runs on the GPU that owns the operands (found from the first operand pointer
 *     and made current for the call) and is enqueued on `stream`, a cudaStream_t of that
 *     GPU passed as an opaque pointer; nothing synchronises the host.
 *   - The library allocates no device memory at run time: scratch comes from the caller
 *     through `workspace`, sized by the matching *_workspace_bytes() query. The one
 *     exception is semx_linoss_bwd_noalloc, which takes no workspace and instead uses an
 *     8 MiB scratch pool compiled into the library (held by every GPU that loads it);
 *     apart from that pool's per-device address, the library keeps no state between
 *     calls.
 *   - The return value is SEMX_OK or one of the SEMX_ERR_* codes; no exception crosses
 *     the ABI. semx_last_error() returns a message for the calling host thread.
 *
 * Names, argument meaning and error behaviour follow the reference's operator API; each
 * declaration cites the reference function it replaces (paths relative to the reference
 * project root).
 */
#ifndef SEMX_H
#define SEMX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SEMX_ABI_VERSION 2

typedef void* semx_stream_t; /* cudaStream_t */

enum semx_status {
  SEMX_OK = 0,
  SEMX_ERR_ABI = 1,          /* struct_size mismatch                                  */
  SEMX_ERR_NULL = 2,         /* a required pointer is NULL                            */
  SEMX_ERR_SHAPE = 3,        /* a size is negative/zero where forbidden, or too large */
  SEMX_ERR_UNSUPPORTED = 4,  /* flag combination or size outside what is compiled     */
  SEMX_ERR_ALIGN = 5,        /* a pointer is not aligned as documented                */
  SEMX_ERR_LAUNCH = 6,       /* the CUDA launch itself failed                         */
  SEMX_ERR_WORKSPACE = 7,    /* workspace pointer NULL while workspace is required    */
  SEMX_ERR_DEVICE = 8        /* an operand is not device memory                       */
};

/* ABI version compiled into the library (== SEMX_ABI_VERSION of this header). */
int semx_abi_version(void);
/* Static message for a status code. */
const char* semx_status_string(int status);
/* Message describing the last failing call made from this host thread ("" if none). */
const char* semx_last_error(void);
/* Number of kernels this library has launched successfully in this process, all host
 * threads and devices together (a monotonically increasing counter). No counterpart in
 * the reference; it lets a caller count the device launches of a region of its own. */
uint64_t semx_launch_count(void);
/* Number of tensor-core completion waits, on the current GPU, that ran out of time in this
 * process (the kernel then stops and leaves the rest of its outputs unwritten); 0 in a
 * healthy run. Synchronises with that GPU. No counterpart in the reference. */
int semx_tc_timeouts(uint32_t* count);

/* ------------------------------------------------------------------------------------
 * LinOSS oscillatory scan.
 *
 *   [y1; y2]_t = [[M11, M12], [M21, M22]] [y1; y2]_{t-1} + [F1; F2]_t,   y_{-1} = 0,
 *   output Y2_t = y2_t (complex), one independent 2x2 real transition per oscillator p.
 *
 * variant SEMX_LINOSS_GENERIC: M11..M22 (P,) and F1, F2 (S,L,P) complex are given.
 *   Replaces linoss_scan_triton (models/linoss/triton.py:276-294) and the sequential
 *   _linoss_recurrence (models/linoss/linoss.py:155-180).
 * variants IM / IMEX / DAMPED_IMEX: the kernel builds M and F = (f1, f2) * Bu from the raw
 *   parameters (steps, A_diag, G_diag), applying the same constraints as LinOSS.forward
 *   (models/linoss/linoss.py:81-116: sigmoid(steps), relu(A_diag), the A-from-G or
 *   G-from-A clamps) and the discretisations _apply_linoss_im / _apply_linoss_imex /
 *   _apply_damped_linoss_imex (models/linoss/linoss.py:183-232). Input is Bu (S,L,P)
 *   complex, the projected input of _project_input (models/linoss/linoss.py:148-152).
 *
 * Forward writes Y2 and, if ckpt != NULL, the state entering every `chunk`-step block
 * and the final state: ckpt (S, ceil(L/chunk) + 1, P, 4) fp32 = (y1.re, y1.im, y2.re,
 * y2.im). Backward (needs the forward's ckpt) rebuilds the states chunk by chunk (IMEX:
 * running the symplectic recurrence backwards from each chunk's end; otherwise, or for
 * oscillators with step^2 A near or above 4, re-running it from the chunk start) and writes
 *   GENERIC: dF1, dF2 (S,L,P) complex and dM (4,P) = dM11, dM12, dM21, dM22;
 *   fused:   dBu (S,L,P) complex and dparams (3,P) = d steps, d A_diag, d G_diag
 *            (d G_diag row written only for DAMPED_IMEX).
 * Parameter gradients are reduced over (S, L) in a fixed order (deterministic).
 * chunk must be a positive multiple of 8 and at most 256.
 * ---------------------------------------------------------------------------------- */
enum semx_linoss_variant {
  SEMX_LINOSS_GENERIC = 0,
  SEMX_LINOSS_IM = 1,
  SEMX_LINOSS_IMEX = 2,
  SEMX_LINOSS_DAMPED_IMEX = 3
};

typedef struct SemxLinossArgs {
  uint32_t struct_size;
  int32_t variant;   /* enum semx_linoss_variant                                  */
  int32_t a_from_g;  /* DAMPED_IMEX: 1 = A clamped into the band set by G (default) */
  int32_t chunk;     /* checkpoint interval / backward recompute block, in steps     */
  int64_t S, L, P;   /* sequences, steps per sequence, oscillators                  */
  /* GENERIC inputs */
  const float* M11;
  const float* M12;
  const float* M21;
  const float* M22;
  const float* F1;   /* (S,L,P) complex */
  const float* F2;   /* (S,L,P) complex */
  /* fused-variant inputs */
  const float* steps;  /* (P,) raw, before sigmoid */
  const float* A_diag; /* (P,) raw                 */
  const float* G_diag; /* (P,) raw, DAMPED_IMEX only */
  const float* Bu;     /* (S,L,P) complex            */
  /* forward outputs */
  float* Y2;   /* (S,L,P) complex */
  float* ckpt; /* (S, ceil(L/chunk) + 1, P, 4) or NULL */
  /* backward */
  const float* dY2; /* (S,L,P) complex */
  float* dF1;       /* GENERIC (S,L,P) complex */
  float* dF2;       /* GENERIC (S,L,P) complex */
  float* dBu;       /* fused (S,L,P) complex   */
  float* dM;        /* GENERIC (4,P)           */
  float* dparams;   /* fused (3,P)             */
  void* workspace;  /* semx_linoss_workspace_bytes() bytes, backward only */
  int32_t reverse;  /* 1: step t of a sequence is element L-1-t of its (L,P) block, i.e.
                       the scan runs backwards in time over the stored order (replaces
                       flipping the input and the output); 0: forward */
} SemxLinossArgs;

size_t semx_linoss_args_size(void);
/* Size of ckpt in bytes for (S, L, P, chunk). */
size_t semx_linoss_ckpt_bytes(int64_t S, int64_t L, int64_t P, int32_t chunk);
/* Scratch the backward needs (per-sequence partial reductions). */
size_t semx_linoss_workspace_bytes(const SemxLinossArgs* args);
int semx_linoss_fwd(const SemxLinossArgs* args, semx_stream_t stream);
int semx_linoss_bwd(const SemxLinossArgs* args, semx_stream_t stream);

/* Backward for callers that cannot allocate device memory. It has no counterpart in the
 * reference. Some hosts must never call cudaMalloc on the thread that drives the scan: a
 * real-time audio process callback (cudaMalloc can synchronise the device and stall past
 * the buffer deadline), or a runtime whose own pool owns all device memory. This entry
 * point does exactly what semx_linoss_bwd does, but ignores args->workspace and uses a
 * scratch pool compiled into the library: SEMX_LINOSS_NOALLOC_SCRATCH_BYTES (8 MiB) of
 * device memory that every GPU which loads the library holds until the process exits.
 * A call whose semx_linoss_workspace_bytes() exceeds the pool returns SEMX_ERR_SHAPE
 * without launching. The caller still passes every input and output (ckpt included).
 * The first call on a device looks up the pool's device address (cudaGetSymbolAddress,
 * once per device) and keeps it for the life of the process; make that first call before
 * any stream capture, and make no call after a cudaDeviceReset of that device in the same
 * process (the reset re-loads the library's device code, and the kept address would no
 * longer be the pool's). Every call shares the one pool and nothing in it needs to start
 * at zero (each call overwrites what it reads, or clears it when L == 0), but calls whose
 * work overlaps on the GPU (different streams, or several host threads) race on it:
 * serialise them. */
#define SEMX_LINOSS_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int semx_linoss_bwd_noalloc(const SemxLinossArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Selective-LRU SISO scan with readout (one bank of N modes per channel).
 *
 *   lam  = exp(delta_nu * (-a + j*(omega + [s *] delta_theta)))          (per t, c, n)
 *   Bu   = gain * (B_re + j B_im)_t * x_t,  gain in {gamma, mamba, zoh}
 *   h_t  = lam_t h_{t-1} + Bu_t,            h_{-1} = h0 (default 0)
 *   y_t  = Re(<C_t, h_t>) [+ <g, |h_t|^2>] + D x_t
 * Replaces fused_selective_lru / _SelectiveLRUScan
 * (models/selective_lru/selective_lru_triton.py:398-577) and the materialised path of
 * SelectiveLRU.forward (models/selective_lru/selective_lru.py:242-276, 590-599).
 *
 * real = 1 selects the real specialisation (omega = delta_theta = B_im = C_im = 0; the
 * pointers for those operands, and every *_im pointer, are ignored): the selective
 * diagonal scan h = exp(-delta_nu a) h + gain B_t x, y = <C_t, h> + D x.
 *
 * Shapes: delta_nu, delta_theta, x, y, dy, d_*: (S,L,C); a, omega, g, s: (C,N);
 * B_*, C_* and their grads: (S,L,N); D: (C); h0_*, hf_*, dhf_*, dh0_*: (S,C,N).
 * Optional inputs: g (envelope readout), s (per-mode detune), h0 (initial state),
 * dy / dhf in the backward (NULL = zero). N <= 32.
 * Forward writes y, hf (if non-NULL) and, if ckpt != NULL, the state entering every
 * `chunk`-step block: ckpt (S, ceil(L/chunk), C, N) complex64 (fp32 when real).
 * Backward needs the forward's ckpt and writes every non-NULL gradient; reductions over
 * channels (dB, dC) and over (S, L) (da, domega, dD, dg, ds) use a fixed order.
 * chunk must be a multiple of 4 in [4, 256].
 * ---------------------------------------------------------------------------------- */
enum semx_input_gain {
  SEMX_GAIN_GAMMA = 0, /* sqrt(max(1 - |lam|^2, 1e-6))        */
  SEMX_GAIN_MAMBA = 1, /* delta_nu                             */
  SEMX_GAIN_ZOH = 2,   /* (lam - 1) / (-a + j*base), exact ZOH */
  SEMX_GAIN_NONE = 3   /* 1 (MIMO only)                        */
};

typedef struct SemxSelectiveLruArgs {
  uint32_t struct_size;
  int32_t real;       /* 1 = real specialisation                 */
  int32_t input_gain; /* enum semx_input_gain (not NONE)         */
  int32_t chunk;      /* checkpoint interval, in steps           */
  int64_t S, L, C, N;
  const float* delta_nu;
  const float* delta_theta;
  const float* a;     /* exp(A_log), > 0 */
  const float* omega;
  const float* B_re;
  const float* B_im;
  const float* C_re;
  const float* C_im;
  const float* x;
  const float* D;
  const float* g;     /* envelope gains or NULL */
  const float* s;     /* detune gains or NULL   */
  const float* h0_re; /* initial state or NULL  */
  const float* h0_im;
  /* forward outputs */
  float* y;
  float* hf_re; /* final state or NULL */
  float* hf_im;
  float* ckpt;
  /* backward inputs */
  const float* dy;
  const float* dhf_re;
  const float* dhf_im;
  /* backward outputs (NULL = not wanted) */
  float* d_delta_nu;
  float* d_delta_theta;
  float* dx;
  float* dB_re;
  float* dB_im;
  float* dC_re;
  float* dC_im;
  float* da;
  float* domega;
  float* dD;
  float* dg;
  float* ds;
  float* dh0_re;
  float* dh0_im;
  void* workspace; /* semx_selective_lru_workspace_bytes(), backward only */
  /* Token layout (all zero: the documented (S,L,X) layout). Every per-step operand,
   * output and gradient is a matrix of S*L token rows; step t of sequence s is row
   *   (s / G) * group_stride + (s % G) * seq_stride + t' * step_stride,
   * t' = reverse ? L-1-t : t, with G = seq_group (0 = 1), group_stride (0 = L) and
   * step_stride (0 = 1). Example: activations laid out (B, T, F, X) scanned along T
   * over the B*F sequences: G = F, group_stride = T*F, seq_stride = 1, step_stride = F
   * (no transposed copy). The map must send the S*L pairs (s, t) to distinct rows below
   * S*L (checked: S % G == 0, S and G below 2^31, and the largest row index; a map that
   * sends two tokens to one row is not detected and gives undefined results, with every
   * access still inside the rows). Checkpoints and the final state keep their
   * documented (sequence-major) layouts. */
  int32_t reverse;
  int64_t seq_group, group_stride, seq_stride, step_stride;
} SemxSelectiveLruArgs;

size_t semx_selective_lru_args_size(void);
size_t semx_selective_lru_ckpt_bytes(const SemxSelectiveLruArgs* args);
size_t semx_selective_lru_workspace_bytes(const SemxSelectiveLruArgs* args);
int semx_selective_lru_fwd(const SemxSelectiveLruArgs* args, semx_stream_t stream);
int semx_selective_lru_bwd(const SemxSelectiveLruArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Plain complex diagonal scan h_t = lam_t h_{t-1} + Bu_t, h_{-1} = 0, on split real /
 * imaginary (S,L,N) fp32 tensors. Replaces selective_scan_triton_real /
 * SelectiveScanRealFunction (models/selective_lru/selective_lru_mimo_triton.py:105-211)
 * and _selective_recurrence (models/selective_lru/selective_lru.py:590-599).
 * Backward takes the forward's h and the upstream gradient dh and writes dlam, dBu.
 * ---------------------------------------------------------------------------------- */
typedef struct SemxComplexScanArgs {
  uint32_t struct_size;
  int32_t reserved;
  int64_t S, L, N;
  const float* lam_re;
  const float* lam_im;
  const float* Bu_re;
  const float* Bu_im;
  float* h_re; /* forward output; backward input */
  float* h_im;
  const float* dh_re;
  const float* dh_im;
  float* dlam_re;
  float* dlam_im;
  float* dBu_re;
  float* dBu_im;
} SemxComplexScanArgs;

size_t semx_complex_scan_args_size(void);
int semx_complex_scan_fwd(const SemxComplexScanArgs* args, semx_stream_t stream);
int semx_complex_scan_bwd(const SemxComplexScanArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * MIMO scan with block-diagonal readout and D skip: for every head h of H heads with
 * Nh modes and Fh channels,
 *   h_t = lam_t h_{t-1} + Bu_t                         (modes h*Nh .. h*Nh+Nh-1)
 *   y_t[h*Fh + f] = sum_n Re(C[h,f,n] h_t[n]) + D[h*Fh + f] x_t[h*Fh + f].
 * lam, Bu, h: (S,L,H*Nh) split re/im; C_re, C_im: (H,Fh,Nh); x, y, dy, dx: (S,L,H*Fh).
 * Replaces fused_selective_lru_mimo / _FusedSelectiveLRUMIMO
 * (models/selective_lru/selective_lru_mimo_triton.py:370-462) and the scan + readout of
 * SelectiveLRUMIMO.forward (models/selective_lru/selective_lru.py:550-574).
 * Forward writes y and the state trajectory h. Backward takes h, dy and optionally dh
 * (a gradient on h from feedthrough terms) and writes dlam, dBu, dx, dC_re, dC_im, dD
 * (dC and dD reduced over (S, L) in a fixed order).
 * ---------------------------------------------------------------------------------- */
typedef struct SemxMimoArgs {
  uint32_t struct_size;
  int32_t reserved;
  int64_t S, L, H, Nh, Fh;
  const float* lam_re;
  const float* lam_im;
  const float* Bu_re;
  const float* Bu_im;
  const float* C_re;
  const float* C_im;
  const float* x;
  const float* D;
  float* y;
  float* h_re; /* forward output; backward input */
  float* h_im;
  const float* dy;
  const float* dh_re; /* optional */
  const float* dh_im;
  float* dlam_re;
  float* dlam_im;
  float* dBu_re;
  float* dBu_im;
  float* dx;
  float* dC_re;
  float* dC_im;
  float* dD;
  void* workspace; /* semx_mimo_workspace_bytes(), backward only */
} SemxMimoArgs;

size_t semx_mimo_args_size(void);
size_t semx_mimo_workspace_bytes(const SemxMimoArgs* args);
int semx_mimo_fwd(const SemxMimoArgs* args, semx_stream_t stream);
int semx_mimo_bwd(const SemxMimoArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Fused SelectiveLRUMIMO layer after its token projections: for every head h of H heads
 * (Nh modes, Fh channels, rank R) and token t, from the projection row `proj` and the
 * input x,
 *   dnu = softplus(proj[dnu_h] + b_nu[h]) * rate_scale,  dth = proj[dth_h] + b_th[h]
 *          (dt_bias = [b_nu (H) | b_th (H)], optional: zero when NULL)
 *   lam[n] = exp(dnu (-a[n] + j (omega[n] + (detune ? s[n] dth : dth)))),  a = exp(A_log)
 *   Bu[n]  = gain[n] (bx[n] + sum_r s_b[r] b_t[r,n])   (bx complex: the static drive
 *            sum_f B[h,n,f] x[h*Fh+f]; the rank write real), gain per input_gain
 *            (GAMMA / MAMBA / ZOH / NONE)
 *   h_t    = lam h_{t-1} + Bu,  h_{-1} = 0
 *   y[f]   = sum_n Re(C[h,f,n] h[n]) + D[h*Fh+f] x[h*Fh+f]
 *            + sum_n env[h,f,n] |h[n]|^2                              (envelope only)
 *            + sum_r s_c[r] Re(sum_n c_t[r,n] h[n]) c_out[h*R+r, f]  (R > 0)
 * proj (S,L,P) columns: [dnu (H) | dth (H) | s_b (H*R) | b_t (H*R*Nh) | s_c (H*R) |
 * c_t (H*R*2Nh, per (h, r) Nh real parts then Nh imaginary parts) | bx (H*2Nh, per (h, n)
 * the real then the imaginary part)], P = 2H + 2H*R + 3H*R*Nh + 2H*Nh. The static input
 * map B (H,Nh,Fh,2) of the reference is therefore a block-diagonal part of the caller's
 * projection weight (rows h*2Nh + 2n + {0: re, 1: im}, columns h*Fh .. h*Fh+Fh-1), and its
 * gradients (dB, and B^H d(bx) in dx) come from the projection's backward: dproj's bx
 * columns hold d(loss)/d(bx).
 * x: (S,L,H*Fh); x and proj are fp32, or bf16 when `bf16` is set; y, dy fp32; dx and
 * dproj have the dtype of x. Parameters fp32: A_log, omega, detune_gain (H,Nh);
 * C (H,Fh,Nh,2); D (H*Fh); c_out (H*R,Fh); env_gain (H,Fh,Nh); dt_bias (2H).
 * Replaces SelectiveLRUMIMO.forward after its projections
 * (models/selective_lru/selective_lru.py:488-587): poles, drive, gain, scan, readout and
 * feedthrough in one pass per (sequence, head). Training forwards store the state at
 * every 16-step block in ckpt (semx_mimo_layer_ckpt_bytes()). Backward recomputes from
 * ckpt and writes dx (the skip part D dy), dproj (for the dt columns the gradient
 * with respect to the biased value, which is also the bias's) and the parameter gradients
 * (reduced over sequences in a fixed order; dA_log is with respect to A_log).
 * ---------------------------------------------------------------------------------- */
typedef struct SemxMimoLayerArgs {
  uint32_t struct_size;
  int32_t input_gain; /* enum semx_input_gain                               */
  int32_t rank;       /* R >= 0                                             */
  int32_t detune;     /* 1: detune_gain given                               */
  int32_t envelope;   /* 1: env_gain given                                  */
  int32_t bf16;       /* 1: x, proj, dproj are bf16                         */
  float rate_scale;
  int32_t reserved;
  int64_t S, L, H, Nh, Fh;
  const void* x;
  const void* proj;
  const float* A_log;
  const float* omega;
  const float* detune_gain;
  const float* C;
  const float* D;
  const float* c_out;
  const float* env_gain;
  const float* dt_bias; /* optional */
  float* y;
  float* ckpt; /* optional in the forward; required by the backward */
  const float* dy;
  void* dx;
  void* dproj;
  float* dA_log;
  float* domega;
  float* ddetune;
  float* dC;
  float* dD;
  float* dc_out;
  float* denv;
  float* d_dt_bias; /* written when dt_bias is given */
  void* workspace;  /* semx_mimo_layer_workspace_bytes(), backward only */
} SemxMimoLayerArgs;

/* ------------------------------------------------------------------------------------
 * Mixer surround, channels-last (replaces the depthwise Conv1d + SiLU and the SiLU gate
 * of MambaStyleMixer.forward, models/mixer.py:82-99). `xz` is the in_proj output with
 * rows of `ld` elements: u = columns [0, C), z = columns [C, 2C).
 *   conv_silu: v[s,t,c] = silu(b[c] + sum_k w[c,k] u[s, t - left + k, c]), u = 0 outside
 *              [0, L) (left = K-1: causal; (K-1)/2: centred, as the reference's padding).
 *              Backward writes du into columns [0, C) of dxz and reduces dw, db over
 *              (S, L) in a fixed order (workspace: semx_conv_silu_workspace_bytes()).
 *   gate_silu: o = y * silu(z); backward writes dy and dz (into columns [C, 2C) of dxz).
 * xz, dxz, o, dout are bf16 when `bf16` is set, else fp32; v, dv, y, dy are fp32.
 * ---------------------------------------------------------------------------------- */
typedef struct SemxConvSiluArgs {
  uint32_t struct_size;
  int32_t K;    /* kernel width, 1..8                          */
  int32_t left; /* taps before t                               */
  int32_t bf16; /* xz / dxz dtype                              */
  int64_t S, L, C, ld;
  const void* xz;
  const float* w;  /* (C, K)          */
  const float* b;  /* (C), may be NULL */
  float* v;        /* (S, L, C)       */
  const float* dv; /* (S, L, C)       */
  void* dxz;
  float* dw; /* (C, K) */
  float* db; /* (C), may be NULL */
  void* workspace;
  /* Token layout of xz, v, dv, dxz: as SemxSelectiveLruArgs (reverse: the convolution's
   * window looks at the following steps of the stored order, i.e. the causal convolution
   * of the time-reversed sequence). */
  int32_t reverse;
  int64_t seq_group, group_stride, seq_stride, step_stride;
} SemxConvSiluArgs;

typedef struct SemxGateSiluArgs {
  uint32_t struct_size;
  int32_t bf16; /* xz, o, dout, dxz dtype */
  int64_t n, C, ld; /* n = S*L rows */
  const float* y;   /* (n, C) */
  const void* xz;
  void* o;          /* (n, C) */
  const void* dout; /* (n, C) */
  float* dy;        /* (n, C) */
  void* dxz;
} SemxGateSiluArgs;

size_t semx_conv_silu_args_size(void);
size_t semx_conv_silu_workspace_bytes(const SemxConvSiluArgs* args);
int semx_conv_silu_fwd(const SemxConvSiluArgs* args, semx_stream_t stream);
int semx_conv_silu_bwd(const SemxConvSiluArgs* args, semx_stream_t stream);
size_t semx_gate_silu_args_size(void);
int semx_gate_silu_fwd(const SemxGateSiluArgs* args, semx_stream_t stream);
int semx_gate_silu_bwd(const SemxGateSiluArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * RMS normalisation over the last dimension with a learned gain (replaces the pre-norm
 * Block's RMSNorm, built by create_block with rms_norm=True, models/mamba_block.py:
 * 335-342; the reference takes the class from mamba_ssm):
 *   y[r, j] = x[r, j] / sqrt(mean_j(x[r, j]^2) + eps) * weight[j]
 * computed in fp32; x, y, dy, dx are bf16 when `bf16` is set, else fp32; weight, rstd
 * (n, the 1 / rms of each row, written by the forward when non-NULL, read by the
 * backward), dweight fp32. Rows of d <= 1024 elements. Backward writes dx and dweight,
 * reduced over rows in a fixed order (workspace: semx_rms_norm_workspace_bytes()).
 * ---------------------------------------------------------------------------------- */
typedef struct SemxRmsNormArgs {
  uint32_t struct_size;
  int32_t bf16;
  float eps;
  int32_t reserved;
  int64_t n, d; /* rows, elements per row */
  const void* x;
  const float* weight;
  void* y;
  float* rstd;
  const void* dy;
  void* dx;
  float* dweight;
  void* workspace;
} SemxRmsNormArgs;

size_t semx_rms_norm_args_size(void);
size_t semx_rms_norm_workspace_bytes(const SemxRmsNormArgs* args);
int semx_rms_norm_fwd(const SemxRmsNormArgs* args, semx_stream_t stream);
int semx_rms_norm_bwd(const SemxRmsNormArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Low-rank selective-step projections of the SelectiveLRU layer (replaces
 * delta_nu = softplus(dt_nu_up(dnu_r)) and delta_theta = dt_theta_up(dth_r),
 * models/selective_lru/selective_lru.py:216-220, and the rate scale on delta_nu):
 *   delta_nu[r, c]    = scale * softplus(sum_k W_nu[c, k] z_nu[r, k] + b_nu[c])
 *   delta_theta[r, c] = sum_k W_th[c, k] z_th[r, k] + b_th[c]
 * z_nu, z_th: rows x rank values at row stride ldz (the dnu_r / dth_r columns of the
 * token projection rows, read in place), bf16 when `bf16` is set, else fp32; W (C, rank),
 * b (C), delta_* (rows, C) fp32, 8-byte aligned when C is even; rank 1..8. Backward
 * (d_delta_nu / d_delta_theta may be NULL: zero) writes dz_* (rows, rank, contiguous, the
 * z dtype), dW_* and db_* (fp32, reduced over rows in a fixed order; workspace:
 * semx_step_proj_workspace_bytes()).
 * ---------------------------------------------------------------------------------- */
typedef struct SemxStepProjArgs {
  uint32_t struct_size;
  int32_t bf16;
  int32_t rank;
  float scale;
  int64_t rows, C, ldz;
  const void* z_nu;
  const void* z_th;
  const float* W_nu;
  const float* b_nu;
  const float* W_th;
  const float* b_th;
  float* delta_nu;
  float* delta_th;
  const float* d_delta_nu;
  const float* d_delta_th;
  void* dz_nu;
  void* dz_th;
  float* dW_nu;
  float* db_nu;
  float* dW_th;
  float* db_th;
  void* workspace;
} SemxStepProjArgs;

size_t semx_step_proj_args_size(void);
size_t semx_step_proj_workspace_bytes(const SemxStepProjArgs* args);
int semx_step_proj_fwd(const SemxStepProjArgs* args, semx_stream_t stream);
int semx_step_proj_bwd(const SemxStepProjArgs* args, semx_stream_t stream);

/* ------------------------------------------------------------------------------------
 * LinOSS readout and D skip (replaces Cy = einsum("fn,btn->btf", C, ys).real, Du = x * D,
 * Cy + Du, models/linoss/linoss.py:118-120):
 *   y[r, h] = sum_p Re(C[h, p] y2[r, p]) + D[h] x[r, h]
 * x, y, dy, dx (rows, H) fp32; y2 (rows, P) complex; C (H, P, 2) fp32 (re, im); D (H);
 * P <= 32. Backward writes dx = D dy and the parameter gradients dC (H, P, 2), dD (H),
 * reduced over rows in a fixed order (workspace: semx_linoss_readout_workspace_bytes());
 * the state gradient dy2 = dy conj(C) (a contraction over channels) is the caller's GEMM.
 * ---------------------------------------------------------------------------------- */
typedef struct SemxLinossReadoutArgs {
  uint32_t struct_size;
  int32_t reserved;
  int64_t rows, H, P;
  const float* x;
  const float* y2;
  const float* C;
  const float* D;
  float* y;
  const float* dy;
  float* dx;
  float* dC;
  float* dD;
  void* workspace;
} SemxLinossReadoutArgs;

size_t semx_linoss_readout_args_size(void);
size_t semx_linoss_readout_workspace_bytes(const SemxLinossReadoutArgs* args);
int semx_linoss_readout_fwd(const SemxLinossReadoutArgs* args, semx_stream_t stream);
int semx_linoss_readout_bwd(const SemxLinossReadoutArgs* args, semx_stream_t stream);

size_t semx_mimo_layer_args_size(void);
size_t semx_mimo_layer_ckpt_bytes(const SemxMimoLayerArgs* args);
size_t semx_mimo_layer_workspace_bytes(const SemxMimoLayerArgs* args);
int semx_mimo_layer_fwd(const SemxMimoLayerArgs* args, semx_stream_t stream);
int semx_mimo_layer_bwd(const SemxMimoLayerArgs* args, semx_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SEMX_H */
