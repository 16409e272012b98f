/*
 * demon_b200.h -- C ABI of the B200 (sm_100a) hot path of the DEMON streaming
 * diffusion engine: NVFP4 quantised linear + fused per-slot ODE step.
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers unless the name says host;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - the library never allocates device memory at run time: callers own every
 *     buffer, except two fixed file-scope device arrays that the library's device
 *     code holds in each device context it is loaded into -- the 8-byte status word
 *     and the demon_nvfp4_noalloc_scratch_bytes() bytes (4.875 MiB) of scratch that
 *     demon_nvfp4_linear_noalloc uses;
 *   - return value 0 = DEMON_OK, otherwise a DEMON_ERR_* code, with a message
 *     retrievable through demon_last_error() (thread-local);
 *   - argument errors are detected on the host before any launch;
 *   - device-side bounded waits that expire set bits in a per-device status
 *     word, read (and cleared) with demon_device_status().
 *
 * The reference has no NVFP4 plugin or op.  Each entry point below names the
 * reference interface it stands in for (file:line in daydreamlive/DEMON).
 */
#ifndef DEMON_B200_H
#define DEMON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DEMON_ABI_VERSION 1

#if defined(__GNUC__)
#define DEMON_API __attribute__((visibility("default")))
#else
#define DEMON_API
#endif

enum {
  DEMON_OK = 0,
  DEMON_ERR_INVALID = 1,     /* bad shape / stride / alignment / null pointer */
  DEMON_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  DEMON_ERR_TIMEOUT = 3,     /* a device-side bounded wait expired */
  DEMON_ERR_UNSUPPORTED = 4  /* device is not sm_100 */
};

/* Global-scale policy of the activation quantiser. */
enum {
  DEMON_GS_STATIC = 0,  /* gs[0] supplied by the caller (calibrated) */
  DEMON_GS_DYNAMIC = 1, /* gs[0] = max(amax(x), 1e-12) / 2688, written (two passes) */
  DEMON_GS_PER_ROW = 2  /* gs[m] = max(amax(x[m,:]), 1e-12) / 2688, written (one pass,
                           batch-invariant: a row's codes never depend on other rows) */
};

DEMON_API int demon_abi_version(void);

/* sizeof(DemonGemmArgs) and sizeof(DemonOdeSlot) as compiled, for binding checks. */
DEMON_API int demon_struct_sizes(int64_t* gemm_args, int64_t* ode_slot);

/* Copies the calling thread's last error message into buf (NUL-terminated). */
DEMON_API int demon_last_error(char* buf, size_t n);

/* Reads the device status word of the current device into out[0..1]
 * (out[0]: DEMON_DEV_* bits, out[1]: first failing site) and clears it.
 * Synchronises `stream`. */
DEMON_API int demon_device_status(unsigned int* out_host, void* stream);

/* Bytes of a block-scale buffer for `rows` x K in the tcgen05 layout
 * (rows padded to 128, K/16 scales per row). */
DEMON_API int64_t demon_nvfp4_sf_bytes(int64_t rows, int64_t K);

/*
 * NVFP4 activation quantiser: bf16 x[M, ldx] -> E2M1 codes[M, K/2] (two per
 * byte, element 2j in the low nibble), E4M3 block scales sf (16-element blocks
 * along K, tcgen05 128x4-chunk layout, demon_nvfp4_sf_bytes(M, K) bytes, pad
 * rows written as zero) and fp32 global scale(s) gs.
 * Stands in for the activation Q node of the reference's quantised linear
 * (acestep/engine/trt/fp8_onnx.py:847-952, per-tensor FP8 W8A8 activations)
 * and its weight quantiser (fp8_onnx.py:115-149).  K % 64 == 0, ldx % 8 == 0.
 */
DEMON_API int demon_nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, int gs_mode, float* gs,
                         uint8_t* codes, uint8_t* sf, void* stream);

/*
 * Block-scaled NVFP4 GEMM with fused epilogue:
 *   acc[m,n] = sum_k a[m,k] * w[n,k]                        (tcgen05, fp32 in TMEM)
 *   y[m,n]   = alpha * (acc[m,n] + lora[m,n]) + bias[n]     alpha = a_gs[m|0] * w_gs[0 | n/128]
 *   lora     = sum_j lora_xa[m,j] * lora_b[n,j]             (tcgen05 bf16 MMA into the same
 *                                                            accumulator; lora_xa comes from
 *                                                            demon_lora_down, already divided
 *                                                            by alpha_m and multiplied by the
 *                                                            strength)
 *   y        = gate[m / gate_rows, n] * y                   (optional AdaLN gate)
 *   out[m,n] = residual[m,n] + y                            (optional), stored as bf16.
 * Stands in for the DiT nn.Linear call sites (acestep/models/modeling_acestep_v15_turbo.py:
 * 286-289, 311-345, 377, 538) plus the gated residual that follows o_proj / MLP
 * (turbo.py:525-546), and for the LoRA writeback W = base + sum s_i B_i A_i
 * (acestep/engine/lora.py:283-366, 811-833) without rewriting W.
 * w_gs_per_block: w_gs holds N/128 scales, one per 128-column block, so that several
 * linears that read the same activation (q/k/v, MLP gate/up) run as one GEMM over their
 * concatenated packed weights while each keeps its own per-tensor scale.
 * Constraints: K % 256 == 0, N % 128 == 0, ldo/ldr % 8 == 0, lora_rank % 16 == 0 and <= 128.
 */
typedef struct DemonGemmArgs {
  const uint8_t* a_codes; /* [M, K/2] */
  const uint8_t* a_sf;    /* demon_nvfp4_sf_bytes(M, K) */
  const float* a_gs;      /* [1] or [M] */
  int32_t a_gs_per_row;
  int32_t w_gs_per_block;
  const uint8_t* w_codes; /* [N, K/2] */
  const uint8_t* w_sf;    /* demon_nvfp4_sf_bytes(N, K) */
  const float* w_gs;      /* [1], or [N/128] with w_gs_per_block */
  int64_t M, N, K;
  void* out;              /* bf16 [M, ldo] */
  int64_t ldo;
  const void* bias;       /* bf16 [N] or NULL */
  const void* residual;   /* bf16 [M, ldr] or NULL (may alias out) */
  int64_t ldr;
  const void* gate;       /* bf16 [M / gate_rows, ld_gate] or NULL */
  int64_t gate_rows;      /* rows per gate row (sequence length) */
  int64_t ld_gate;
  const void* lora_xa;    /* bf16 [M, lora_rank] or NULL */
  const void* lora_b;     /* bf16 [N, lora_rank] */
  int64_t lora_rank;
  /* Per-head RMSNorm (+ rotary embedding) of the output, for q/k projections: output columns
   * [0, hn_cols) form heads of 128; a head in [0, hn_q_cols) is normalised with weight hn_wq,
   * the others with hn_wk (bf16 [128] each): y = bf16(w * bf16(y * rsqrt(mean(y^2) + hn_eps))),
   * then, with rope_cos / rope_sin (bf16 [rope_S, 128], position = row % rope_S),
   * y = bf16(bf16(y * cos) + bf16(rotate_half(y) * sin)) -- the q_norm / k_norm and
   * apply_rotary_pos_emb of AceStepAttention.forward (turbo.py:311-345).  hn_cols = 0: off.
   * Needs N % 256 == 0, no gate / residual. */
  int64_t hn_cols, hn_q_cols, rope_S;
  const void* hn_wq;
  const void* hn_wk;
  const void* rope_cos;
  const void* rope_sin;
  float hn_eps;
  /* SwiGLU epilogue (silu_mul != 0): the weight's rows are gate and up blocks of 128
   * interleaved (gate 0..127, up 0..127, gate 128..255, ...; nvfp4.interleave_weights), and
   * the output is h = bf16(bf16(silu(g)) * u) of width N / 2 (out [M, ldo >= N / 2]) with
   * g, u = bf16(alpha * acc + bias) of the paired columns -- Qwen3MLP's
   * act_fn(gate_proj(x)) * up_proj(x) (turbo.py:34-35), bit-identical to
   * demon_silu_mul_quantize's h.  Needs N % 256 == 0; excludes LoRA, head norm, gate,
   * residual. */
  int32_t silu_mul;
  /* rope_half != 0: the caller guarantees that columns 64..127 of rope_cos / rope_sin equal
   * columns 0..63 (the standard rotate-half embedding, cat(freqs, freqs)); only the first 64
   * columns are read, and the epilogue stages half the table (a faster kernel form). */
  int32_t rope_half;
} DemonGemmArgs;

DEMON_API int demon_nvfp4_gemm(const DemonGemmArgs* args, void* stream);

/*
 * Test hook for the bounded device-side waits (no counterpart in the reference): arms the
 * next demon_nvfp4_gemm launch made by the calling thread.  In that launch the first CTA
 * (CTA pair) waits at most wait_ns of device time per wait, and its first CTA never issues
 * the loads of its first pipeline stage, so the MMA issuer's wait on that stage runs out.
 * The CTA then records DEMON_DEV_TIMEOUT in the status word (demon_device_status), stops
 * issuing, waits (bounded) for the copies it issued, frees its tensor memory and returns;
 * the other CTAs finish normally.  The output of the armed launch is undefined; later
 * launches are unaffected.  wait_ns in [1e5, 1e9], or 0 to disarm.
 */
DEMON_API int demon_test_arm_gemm_stall(int64_t wait_ns);

/*
 * LoRA down-projection for the fused epilogue (tcgen05 bf16 GEMM):
 *   xa[m, j] = col_scale[j] * sum_k x[m,k] * lora_a[j,k] / (a_gs[m|0] * w_gs[0])
 * x bf16 [M, ldx], lora_a bf16 [rank, K] (PEFT lora_A layout, acestep/engine/lora.py:294-302),
 * col_scale fp32 [rank] (the strength of the LoRA each rank column belongs to),
 * xa bf16 [M, rank].  K % 64 == 0, rank % 16 == 0, rank <= 128.
 */
DEMON_API int demon_lora_down(const void* x, int64_t M, int64_t K, int64_t ldx, const void* lora_a, int64_t rank,
                    const float* col_scale, const float* a_gs, int a_gs_per_row, const float* w_gs, void* xa,
                    void* stream);

/*
 * bf16 linear on the tensor cores (tcgen05 kind::f16, fp32 accumulate, one rounding):
 *   out[m, n] = bf16(sum_k x[m,k] * w[n,k] + bias[n])
 * x bf16 [M, ldx], w bf16 [N, K] (nn.Linear layout), bias bf16 [N] or NULL, out bf16 [M, ldo].
 * For the DiT projections the reference keeps in bf16: proj_in (Conv1d, kernel = stride =
 * patch, as a linear over patches), proj_out (ConvTranspose1d likewise) and the timestep
 * embedding MLPs (acestep/models/modeling_acestep_v15_turbo.py:207-261, 1262-1307).  Every
 * output row depends on its own input row only (fixed tile shape and summation order), so a
 * slot's result does not depend on the batch it is computed in.
 * K % 64 == 0, N % 64 == 0, ldx/ldo % 8 == 0.
 */
DEMON_API int demon_bf16_linear(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w, int64_t N,
                                const void* bias, void* out, int64_t ldo, void* stream);

/*
 * DiT row kernels around the NVFP4 GEMMs.  Every output row is computed by a fixed set of
 * lanes in a fixed order, independent of M, so results do not depend on the batch.
 *
 * demon_adanorm_quantize: per row of x bf16 [M, D]
 *   y = bf16(bf16(bf16(norm_w * bf16(x * rsqrt(mean(x^2) + eps))) * scale1[b]) + shift[b]),
 *   b = m / rows_per_mod, scale1 = 1 + scale (bf16 [B, ld_mod]; NULL skips the product,
 *   shift NULL skips the sum), then NVFP4-quantised with a per-row global scale into
 *   codes / sf / gs (NULL codes: no quantisation) and/or stored as bf16 into y [M, ldy].
 *   Stands in for Qwen3RMSNorm + the AdaLN modulation of AceStepDiTLayer.forward and the
 *   output norm of AceStepDiTModel.forward (acestep/models/modeling_acestep_v15_turbo.py:
 *   508-510, 522, 531-538, 1495-1500) followed by the activation quantiser.
 *   D in {256, 512, 1024, 2048, 3072, 4096, 6144, 8192}.
 * demon_silu_mul_quantize: gu bf16 [M, ld] holds gate in columns [0, F) and up in [F, 2F);
 *   h = bf16(bf16(silu(gate)) * up), NVFP4-quantised per row (Qwen3MLP's act_fn(gate) * up,
 *   turbo.py:34-35) and, when y is given, also stored as bf16 into y [M, ldy].  F as D above.
 * demon_head_norm_rope: in place on `heads` heads of 128 columns starting at col0 of
 *   x bf16 [M, ld]: Qwen3RMSNorm over each head (weight w [128]), then, when cos/sin
 *   (bf16 [S, 128], position = m % S) are given, x * cos + rotate_half(x) * sin with each
 *   product and the sum rounded to bf16 (q_norm / k_norm and apply_rotary_pos_emb in
 *   AceStepAttention.forward, turbo.py:311-345).
 */
DEMON_API int demon_adanorm_quantize(const void* x, int64_t M, int64_t D, int64_t ldx, const void* norm_w,
                                     const void* scale1, const void* shift, int64_t rows_per_mod, int64_t ld_mod,
                                     float eps, float* gs, uint8_t* codes, uint8_t* sf, void* y, int64_t ldy,
                                     void* stream);
DEMON_API int demon_silu_mul_quantize(const void* gu, int64_t M, int64_t F, int64_t ld, float* gs, uint8_t* codes,
                                      uint8_t* sf, void* y, int64_t ldy, void* stream);
DEMON_API int demon_head_norm_rope(void* x, int64_t M, int64_t ld, int64_t col0, int64_t heads, const void* w,
                                   const void* cos, const void* sin, int64_t S, float eps, void* stream);

/*
 * NVFP4 linear that allocates nothing: out = x W^T + bias (bf16 [M, ldo]),
 * i.e. demon_nvfp4_quantize (per-row global scales) followed by
 * demon_nvfp4_gemm, with the quantised activation kept in a fixed device
 * array inside the library instead of caller buffers.  No counterpart in the
 * reference: it is for callers that cannot allocate device memory while the
 * layer runs (a TensorRT plugin's enqueue(), a real-time thread that must not
 * block in cudaMalloc).  Limits: M * K <= 8,388,608, M <= 65,536, K % 256 == 0,
 * N % 128 == 0.  Every argument check of both kernels runs before the first
 * launch, so a rejected call launches nothing.  The array
 * (demon_nvfp4_noalloc_scratch_bytes() bytes) is set up in a device's context
 * when the library's device code is first loaded there (at the latest on the
 * first call on that device) and stays until the context ends; it is shared
 * by all calls on a device: calls that overlap on the GPU race.  The first
 * call on a device looks up the array's address, which may also load the
 * module: make it before any stream capture.
 */
DEMON_API int64_t demon_nvfp4_noalloc_scratch_bytes(void);
DEMON_API int demon_nvfp4_linear_noalloc(const void* x, int64_t M, int64_t K, int64_t ldx, const uint8_t* w_codes,
                                         const uint8_t* w_sf, const float* w_gs, int64_t N, const void* bias,
                                         void* out, int64_t ldo, void* stream);

/*
 * Fused per-slot ODE step over one tick (all slots in one launch).
 * Stands in for StreamPipeline._tick_pt's post-forward section
 * (acestep/engine/stream.py:983-998, 1060-1276) composed from
 * acestep/engine/ode_steps.py:72-392 (x0_from_vel, mask_pre_blend,
 * mask_post_blend_x0, blend_x0_target, blend_velocities, step_ode_euler,
 * step_sde_curve, step_sde_renoise, MomentumBuffer, apg_forward, cfg_rescale).
 * All latents are bf16 [T, D] row-major with D == 64; curves are fp32 [T].
 * A NULL curve pointer means "use the scalar field next to it".
 */
enum {
  DEMON_ODE_X0PATH = 1 << 0,      /* x0-blend integration (needs_x0 in stream.py:1188-1194) */
  DEMON_ODE_MASK = 1 << 1,        /* latent mask: pre-blend base, post-blend x0 */
  DEMON_ODE_CFG = 1 << 2,         /* APG guidance (apg_forward) */
  DEMON_ODE_MOM_INIT = 1 << 3,    /* momentum running average starts at 0 */
  DEMON_ODE_RESCALE = 1 << 4,     /* cfg_rescale */
  DEMON_ODE_X0_TARGET = 1 << 5,   /* x0 = (1-c) x0 + c * x0_target */
  DEMON_ODE_FINAL = 1 << 6,       /* t_next <= 0 */
  DEMON_ODE_SDE_CURVE = 1 << 7,   /* step_sde_curve */
  DEMON_ODE_SDE_BARE = 1 << 8,    /* step_sde_renoise */
  DEMON_ODE_ONC = 1 << 9,         /* ode_noise_curve injection */
  DEMON_ODE_CACHE_NEG = 1 << 10,  /* write v_neg into neg_cache (RCFG initialize, step 0) */
  DEMON_ODE_DEC_OUT = 1 << 11,    /* write next tick's decoder input */
  DEMON_ODE_DEC_MASK = 1 << 12,   /* next decoder input is mask-pre-blended */
  DEMON_ODE_VS = 1 << 13,         /* velocity_scale present */
  DEMON_ODE_DCW_LO = 1 << 14,     /* DCW: correct the haar low band (dcw_lo = t * scaler per band) */
  DEMON_ODE_DCW_HI = 1 << 15,     /* DCW: correct the haar high band (dcw_hi = (1 - t) * scaler) */
  DEMON_ODE_DCW_PIX = 1 << 16     /* DCW pix mode: x + s (x - denoised) per frame (s = dcw_lo) */
};

#define DEMON_ODE_MAX_COND 4

typedef struct DemonOdeSlot {
  void* xt;                                    /* in: state x_t; out: x_{t_next} (in place) */
  const void* v_pos[DEMON_ODE_MAX_COND];       /* positive velocities, one per active condition */
  const float* w_pos[DEMON_ODE_MAX_COND];      /* temporal weights [T] (NULL = 1) */
  const void* v_neg[DEMON_ODE_MAX_COND];       /* negative velocities (forward, cache or initial noise) */
  const float* w_neg[DEMON_ODE_MAX_COND];
  int32_t n_pos, n_neg;
  void* neg_cache;                             /* RCFG initialize cache (written with CACHE_NEG) */
  void* momentum;                              /* APG running average [T, D] (in/out) */
  const float* guidance; float guidance_s;     /* APG guidance scale */
  const float* apg_mom; float apg_mom_s;       /* APG momentum */
  const float* rescale; float rescale_s;       /* cfg_rescale blend */
  const float* vscale; float vscale_s;         /* velocity_scale */
  const float* sdc; float sdc_s;               /* sde_denoise_curve */
  const float* onc; float onc_s;               /* ode_noise_curve */
  const float* x0_coef; float x0_coef_s;       /* x0_target blend coefficient (times x0_coef_mul) */
  float x0_coef_mul;
  float mask_s;                                /* mask strength at this step */
  const float* mask;                           /* [T] latent mask (1 = generate) */
  const void* mask_orig;                       /* [T, D] original latents */
  const void* mask_noise;                      /* [T, D] fixed mask noise */
  const void* source;                          /* [T, D] source latents (SDE curve) */
  const void* x0_target;                       /* [T, D] */
  const void* noise;                           /* [T, D] step noise (NULL = in-kernel counter-based noise) */
  void* dec_out;                               /* [T, D] next decoder input */
  float mask_s_next;                           /* mask strength at the next step */
  float t_curr, t_next;
  int32_t flags;
  uint64_t seed;                               /* key of the in-kernel noise */
  uint64_t step;                               /* step index in the noise counter */
  /* DCW post-step correction (StreamPipeline._maybe_dcw, stream.py:1387-1405;
   * DCWCorrector.apply, dcw.py:428-490): band coefficients per haar band k = t / 2
   * ([ceil(T / 2)] fp32, the scaler curves already multiplied by t / (1 - t) and resampled),
   * or per frame ([T]) in pix mode; NULL = the scalar next to it. */
  const float* dcw_lo; float dcw_lo_s;
  const float* dcw_hi; float dcw_hi_s;
} DemonOdeSlot;

/*
 * slots: device array of n_slots DemonOdeSlot (the library reads it on the device);
 * gain: bf16 [T, D] channel gain applied to the next decoder input (NULL = 1);
 * T: frames per slot (all slots share T, as StreamPipeline.tick enforces,
 * stream.py:867-883); D must be 64.
 */
DEMON_API int demon_ode_step(const DemonOdeSlot* slots_dev, int32_t n_slots, int64_t T, int64_t D, const void* gain,
                   void* stream);

/*
 * Decoder-input preparation for newly initialised slots (stream.py:983-998):
 * dec_out = (mask ? mask_pre_blend(xt) : xt) * gain, per slot, using
 * t_curr / mask_s / DEMON_ODE_MASK of each slot descriptor.
 */
DEMON_API int demon_ode_prepare(const DemonOdeSlot* slots_dev, int32_t n_slots, int64_t T, int64_t D, const void* gain,
                      void* stream);

/*
 * CTAs per slot cluster that demon_ode_step / demon_ode_prepare launch for n_slots slots of
 * T frames on the current device: 16 while the CTAs need at most one per SM, else 8 while all
 * clusters of 8 are resident at once, else 4.  Launches nothing (for tests and tuning).
 */
DEMON_API int demon_ode_cluster_size(int32_t n_slots, int64_t T, int32_t* cluster);

/*
 * Bidirectional grouped-query attention, head_dim 128, bf16:
 *   o[b, i, h] = sum_j softmax_j(scale * q[b, i, h] . k[b, j, h / G]) v[b, j, h / G],
 * G = Hq / Hk (even), j over all L keys, or over |i - j| <= window when window >= 0 (then
 * S == L).  Element (b, i, h, d) of q sits at q + b * sq + i * ldq + h * 128 + d (pitches in
 * elements; heads contiguous within a row), likewise k / v (Hk heads, L rows) and o (Hq heads,
 * S rows); the q / k / v pitches of one fused projection output work as they are.
 * Stands in for the attention interface call of AceStepAttention.forward
 * (acestep/models/modeling_acestep_v15_turbo.py:358-372), the sliding-window band of
 * lines 110-112 of the same file, with the GQA K / V heads shared instead of repeated.
 * fp32 scores and softmax, bf16 probabilities into the P V product; each (sequence, head,
 * query block) is computed from that sequence alone (no split over keys), so results do
 * not depend on the batch.  Limits (DEMON_ERR_INVALID otherwise): S, L < 2^30 and
 * B * Hq / 2 * ceil(S / 128) < 2^31 work units.
 */
typedef struct DemonAttnArgs {
  const void* q;
  int64_t ldq, sq;
  const void* k;
  int64_t ldk, sk;
  const void* v;
  int64_t ldv, sv;
  void* o;
  int64_t ldo, so;
  int32_t B, S, L, Hq, Hk, head_dim, window; /* window -1: no band */
  float scale;                              /* softmax scale, e.g. 1 / sqrt(128) */
} DemonAttnArgs;

DEMON_API int demon_attention(const DemonAttnArgs* args, void* stream);
DEMON_API int64_t demon_attention_args_size(void);

#ifdef __cplusplus
}
#endif
#endif /* DEMON_B200_H */
