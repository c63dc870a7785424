// Kernel ids, per-kernel plan-parameter slots and host launchers.
// The plan emitter (plan.py) writes the same slot numbers; keep both in sync
// (tests/test_plan.py checks the Python mirror against this header).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "plan_format.h"

namespace emx {

enum KernelId : uint32_t {
  K_PAD_NHWC = 1,       // NCHW 8-bit -> zero-bordered chunk-planar NHWC (optionally XOR 0x80)
  K_QCONV_TC = 2,       // QLinearConv implicit GEMM on tcgen05 kind::i8 (+ fused QLinearAdd)
  K_QCONV_GENERIC = 3,  // QLinearConv, any stride/pad/dilation/group, CUDA cores
  K_QLINEAR_ADD = 4,    // com.microsoft QLinearAdd, same-shape operands
  K_GEMM_F32 = 5,       // Gemm fp32, reference accumulation order (+bias, +Relu)
  K_RELU_F32 = 6,
  K_NBITS_GEMM = 7,     // MatMulNBits int4 x fp16 on tcgen05 kind::f16 (+ fused Swish*Mul of a gate/up pair)
  K_SWISH_F16 = 8,
  K_MUL_F16 = 9,
  K_ATTENTION_F16 = 10, // opset-23 Attention in the reference's fp16 arithmetic
  K_LSTM_F32 = 11,      // LSTM forward, reference accumulation order (1 + 1 + T launches)
  K_QLINEAR_MATMUL = 13,
  K_MATMUL_INTEGER = 14,
  K_CONV_F32 = 15,
  K_SOFTMAX_F32 = 16,
  K_QUANTIZE_LINEAR = 17,
  K_DEQUANTIZE_LINEAR = 18,
  K_ATTENTION_TC = 19,  // opset-23 Attention, fast mode: tcgen05 kind::f16, fp32 online softmax (attention_tc.cu)
  K_COPY = 20,             // byte copy (a Reshape whose output is a graph output)
  K_TRANSPOSE = 21,        // N-d transpose, 1/2/4-byte elements
  K_MAXPOOL = 22,          // 2-D MaxPool, 8-bit
  K_QLINEAR_AVGPOOL = 23,  // com.microsoft QLinearAveragePool, 2-D NCHW, 8-bit
  K_QLINEAR_SOFTMAX = 24,  // com.microsoft QLinearSoftmax, 8-bit
  K_NBITS_I8 = 25,         // MatMulNBits accuracy_level 4: int8 activations, exact block sums (nbits_i8.cu)
};

// Chunk-planar zero-bordered layout ("planar" below): [C/16][rows][16 bytes],
// row = n*Hp*Wp + hp*Wp + wp, `*_ROWS` rows allocated per plane (>= N*Hp*Wp
// plus a tail the conv windows may read).

// ---- K_PAD_NHWC: t[0]=x (NCHW), t[1]=y (planar)
enum { PAD_N, PAD_C, PAD_H, PAD_W, PAD_TOP, PAD_LEFT, PAD_HP, PAD_WP, PAD_XOR, PAD_ROWS };

// ---- K_QCONV_TC: t[0]=x (planar), t[1]=w image, t[2]=epilogue table
//      (float scale[OC], int32 bias[OC]), t[3]=residual (planar) or -1, t[4]=y,
//      t[5]=fused-add table [conv byte][residual byte] -> output byte, or -1
enum {
  QC_N, QC_CIN, QC_OC, QC_KH, QC_KW, QC_HP, QC_WP, QC_OH, QC_OW, QC_A_SIGNED, QC_Y_ZERO,
  QC_Y_LAYOUT /*0 planar, 1 NCHW*/, QC_Y_XOR, QC_Y_HP, QC_Y_WP, QC_Y_PT, QC_Y_PL, QC_Y_SIGNED,
  QC_HAS_ADD, QC_C_ZERO /*conv-side zero in the add*/, QC_R_ZERO, QC_R_XOR, QC_R_SIGNED, QC_R_HP, QC_R_WP,
  QC_R_PT, QC_R_PL, QC_ADD_ZERO /*add output zero*/, QC_ADD_SIGNED, QC_X_ROWS, QC_Y_ROWS, QC_R_ROWS,
  QC_CHAIN /*first op of a chain: its length L (t[6] = chain state); later members: -1; else 0*/,
  QC_RQ_INT /*1: |(float)acc * scale| < 2^21 for every accumulator the weights allow (planner-proved), so
               rint + zero point + clamp run as one integer saturating pack, exactly*/
};
enum { QCF_C_SCALE, QCF_R_SCALE, QCF_ADD_SCALE };

// ---- K_QCONV_GENERIC: t[0]=x NCHW, t[1]=w OIHW, t[2]=w_scale f32, t[3]=w_zero i32|-1,
//      t[4]=bias i32|-1, t[5]=y NCHW
enum {
  QG_N, QG_C, QG_H, QG_W, QG_OC, QG_KH, QG_KW, QG_OH, QG_OW, QG_SH, QG_SW, QG_PT, QG_PL, QG_DH, QG_DW,
  QG_GROUP, QG_X_SIGNED, QG_W_SIGNED, QG_Y_SIGNED, QG_X_ZERO, QG_Y_ZERO, QG_WS_PER_CH, QG_WZ_PER_CH
};
enum { QGF_X_SCALE, QGF_Y_SCALE };

// ---- K_QLINEAR_ADD: t[0]=a, t[1]=b, t[2]=y
enum { QA_COUNT, QA_A_SIGNED, QA_B_SIGNED, QA_Y_SIGNED, QA_A_ZERO, QA_B_ZERO, QA_Y_ZERO, QA_BATCH };
enum { QAF_A_SCALE, QAF_B_SCALE, QAF_Y_SCALE };

// ---- K_GEMM_F32: t[0]=A, t[1]=B, t[2]=bias|-1, t[3]=Y
enum { GM_M, GM_N, GM_K, GM_TRANS_A, GM_TRANS_B, GM_BIAS_MODE, GM_RELU };
enum { GMF_ALPHA, GMF_BETA };

// ---- K_NBITS_GEMM: t[0]=A f16 [rows][a_pitch], t[1]=weight image (see nbits.cu),
//      t[2]=bias f32 [n_tiles*128] | -1, t[3]=Y f16 [rows][y_pitch]
enum {
  NB_ROWS, NB_K, NB_N_OUT, NB_KSTEPS, NB_NTILES, NB_GROUPS, NB_FUSED, NB_A_PITCH, NB_Y_PITCH, NB_ROWS_PER_BATCH,
  NB_ROUNDED_DEQUANT /*1: one MMA per K slice on fp16-rounded weights (default 0: exact hi + lo)*/
};
enum { NBF_ALPHA };

// ---- K_NBITS_I8: t[0]=A f16 [rows][K], t[1]=weights int8 (q - zp) [N][KP] (zero past K),
//      t[2]=scales f32 [N][NBLK], t[3]=bias f32 [N] | -1, t[4]=scratch int8 [rows][KP] (quantised A),
//      t[5]=scratch f32 [rows][NBLK] (A's block scales), t[6]=Y f16 [rows][N]; KP = NBLK * BLOCK
enum { NI_ROWS, NI_K, NI_KP, NI_N, NI_BLOCK, NI_NBLK, NI_ROWS_PER_BATCH };

// ---- K_ATTENTION_F16 and K_ATTENTION_TC (same slots; the latter needs head sizes of 128 and
//      ignores t[4]): t[0]=Q, t[1]=K, t[2]=V, t[3]=Y (fp16), t[4]=scratch (4 words);
//      element (b, h, t, d) of a tensor sits at b*SB + h*SH + t*ST + d (3-D or 4-D layouts)
enum {
  AT_B, AT_HQ, AT_GROUP, AT_TQ, AT_TK, AT_PAST, AT_D, AT_DV, AT_CAUSAL,
  AT_Q_SB, AT_Q_SH, AT_Q_ST, AT_K_SB, AT_K_SH, AT_K_ST, AT_V_SB, AT_V_SH, AT_V_ST, AT_O_SB, AT_O_SH, AT_O_ST
};
enum { ATF_SCALE };

// ---- K_LSTM_F32: t[0]=X [T][B][I], t[1]=W rows interleaved [4Hp][I] (g = i,o,f,c; see below),
//      t[2]=R interleaved [4Hp][H], t[3]=Wb+Rb interleaved [4Hp], t[4]=scratch [T*B][4Hp],
//      t[5]=scratch h [2][B][H], t[6]=scratch c [B][H], t[7]=Y|-1, t[8]=Y_h|-1, t[9]=Y_c|-1
//      gate columns are in tiles of 4 * LS_TILE_UNITS: position g * LS_TILE_UNITS + u of tile T is
//      gate g of unit T * LS_TILE_UNITS + u (units padded to a multiple of LS_TILE_UNITS with zero rows)
enum { LS_T, LS_B, LS_I, LS_H, LS_GX_PLACEHOLDER /*1: t[4] is a placeholder (persistent path planned)*/ };
enum { LS_TILE_UNITS = 16 };
// Persistent LSTM kernel (lstm.cu): chunk of K staged per cp.async stage, stages,
// batch rows per thread (max), threads per CTA (max), shared memory per CTA,
// and the SM count the planner assumes when it leaves out the x-partials scratch.
// (The shared-memory limit is dynamic memory: 225 KB, below the 227 KB a CTA may
// hold in total, which also covers the kernel's static words.)
enum { LP_KC = 8, LP_STAGES = 6, LP_RB_MAX = 4, LP_MAX_THREADS = 512, LP_SMEM_LIMIT = 230400, LP_PLAN_SMS = 148 };

// ---- K_COPY: t[0]=src, t[1]=dst; CP_BATCH > 0: CP_BYTES covers that many batch entries
enum { CP_BYTES, CP_BATCH };

// ---- K_TRANSPOSE: t[0]=x, t[1]=y; y[o0..o5] = x[sum o_i * TR_S_i] over the output dims
//      (rank padded to 6 with leading 1s; TR_S_i = x's stride of the input axis perm[i]);
//      TR_BATCH_AXIS: padded output axis that follows the run's batch (batched plans)
enum { TR_ELEM, TR_D0, TR_D1, TR_D2, TR_D3, TR_D4, TR_D5, TR_S0, TR_S1, TR_S2, TR_S3, TR_S4, TR_S5, TR_BATCH_AXIS };

// ---- K_MAXPOOL / K_QLINEAR_AVGPOOL: t[0]=x NCHW, t[1]=y NCHW
enum {
  PL_N, PL_C, PL_H, PL_W, PL_OH, PL_OW, PL_KH, PL_KW, PL_SH, PL_SW, PL_DH, PL_DW, PL_PT, PL_PL, PL_X_SIGNED,
  PL_Y_SIGNED, PL_COUNT_PAD, PL_X_ZERO, PL_Y_ZERO
};
enum { PLF_SCALE /*QLinearAveragePool: (float)x_scale / (float)y_scale*/ };

// ---- K_QLINEAR_SOFTMAX: t[0]=x, t[1]=y, t[2]=expf table f32 [256][256] (raw byte of the element,
//      raw byte of the row maximum); rows (outer, inner) of axis_size elements at stride inner
enum { QS_OUTER, QS_AXIS, QS_INNER, QS_X_SIGNED, QS_Y_SIGNED, QS_X_ZERO, QS_Y_ZERO };
enum { QSF_X_SCALE, QSF_Y_INV /*floorf(1 / (float)y_scale)*/ };

// ---- K_QLINEAR_MATMUL / K_MATMUL_INTEGER: t[0]=A [M][K] 8-bit, t[1]=B [K][N] 8-bit, t[2]=Y;
//      tensor-core plans add t[3]=B^T [N][K] u8, t[4]=B's column sums [N] i32, t[5]=A's row sums [M] i32
//      (scratch); with QM_B_PACKED (B an initializer) t[3] and t[4] are weights packed by the planner,
//      otherwise scratch the run fills
enum {
  QM_M, QM_K, QM_N, QM_A_SIGNED, QM_B_SIGNED, QM_A_ZERO, QM_B_ZERO, QM_QUANTIZED, QM_USE_INT, QM_FRAC_BITS,
  QM_MULT, QM_Y_ZERO, QM_Y_SIGNED, QM_ROWS_PER_BATCH, QM_B_PACKED
};
enum { QMF_SCALE };

// ---- K_CONV_F32: t[0]=X NCHW, t[1]=W OIHW, t[2]=bias|-1, t[3]=Y
enum {
  CF_N, CF_C, CF_H, CF_W, CF_OC, CF_KH, CF_KW, CF_OH, CF_OW, CF_SH, CF_SW, CF_PT, CF_PL, CF_DH, CF_DW, CF_GROUP,
  CF_ZERO_TAPS_OK  // 1: out-of-image taps may be added as x = 0 (finite weights, no -0 bias)
};

// ---- K_SOFTMAX_F32: t[0]=X, t[1]=Y; shape viewed as [outer][axis][inner]
enum { SM_OUTER, SM_AXIS, SM_INNER, SM_OUTER_PER_BATCH };

// ---- K_QUANTIZE_LINEAR / K_DEQUANTIZE_LINEAR: t[0]=X, t[1]=scale f32 [axis_len], t[2]=zero point|-1, t[3]=Y
enum { QL_COUNT, QL_AXIS_LEN, QL_INNER, QL_SIGNED, QL_ROWS };

// ---- elementwise (K_RELU_F32, K_SWISH_F16, K_MUL_F16): t[0]=x, (t[1]=x2), then y;
//      K_SWISH_F16 may add t[2] = 65536-entry fp16 table (arena, filled at load: Swish of every fp16 value)
enum { EW_COUNT, EW_ROWS /*compiled rows along axis 0 (0: not batched)*/ };
enum { EWF_ALPHA };

struct OpState;

struct LaunchCtx {
  cudaStream_t stream;
  int* d_error;     // device error word
  int64_t batch;    // rows along axis 0 this run (== plan batch unless sliced); 0: plan not batched
  int num_sms;
  // the plan's ops and their states, and this op's index: lets an op launch
  // the ops that follow it together (a chain); null outside a plan
  const PlanOp* ops = nullptr;
  const OpState* states = nullptr;
  size_t n_ops = 0;
  size_t index = 0;
  int fault = 0;  // test hooks in effect (FAULT_* bits, emx_b200_set_fault)
};

// Failure-detection test hooks (emx_b200_set_fault): each makes a bounded
// device wait run out; none faults, traps or hangs the GPU.
enum FaultHook : int {
  FAULT_DROP_CHAIN_PROGRESS = 1,  // chained convolutions never publish their progress words
};

// Last integer slot of every op: 1 when the op's leading (batch) extent
// follows the run's batch slice.  The plan emitter sets it only on ops whose
// leading extent is the plan batch, and marks a plan sliceable only if every
// op that touches activations has it.
constexpr int IP_BATCHED = EMX_OP_MAX_IPARAMS - 1;

// Batch an op processes this run: the run's slice for batched ops of a
// batched plan, else the op's compiled extent.
inline int64_t eff_batch(const LaunchCtx& c, const PlanOp& op, int64_t compiled) {
  return (c.batch > 0 && op.ip[IP_BATCHED]) ? c.batch : compiled;
}

// Launch with programmatic stream serialisation allowed (see pdl_wait() in
// tc100.cuh): every kernel of the library goes through this helper and waits
// on its predecessor inside the kernel.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Opaque per-op state prepared once at plan load (tensor maps, chosen variant).
struct alignas(64) OpState {
  unsigned char bytes[512];
};

// Each kernel family: prepare (load time, may fail with a message) + launch.
typedef int (*PrepareFn)(const PlanOp& op, void* const* ptrs, OpState* st, int device, char* msg, size_t msg_len);
typedef int (*LaunchFn)(const PlanOp& op, void* const* ptrs, const OpState* st, const LaunchCtx& ctx,
                        int* launches);

int prepare_qconv_tc(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_qconv_tc(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_pad_nhwc(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_qconv_generic(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_qlinear_add(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_gemm_f32(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_gemm_f32(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
void launch_hold(const int* flag, int seq, int* err, cudaStream_t stream);
int launch_relu_f32(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_nbits(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_nbits(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_nbits_i8(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_nbits_i8(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_swish_f16(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_swish_f16(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_mul_f16(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_lstm_f32(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_lstm_f32(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
struct QMatMulParams;
int prepare_qmatmul(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_qmatmul(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_qgemm_tc();
int launch_qgemm_tc(const PlanOp&, void* const*, const LaunchCtx&, const QMatMulParams&, int*);
int launch_conv_f32(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_softmax_f32(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_quant(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_attention(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_attention(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_copy(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_transpose(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_maxpool(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_qlinear_avgpool(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int launch_qlinear_softmax(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);
int prepare_attention_tc(const PlanOp&, void* const*, OpState*, int, char*, size_t);
int launch_attention_tc(const PlanOp&, void* const*, const OpState*, const LaunchCtx&, int*);

}  // namespace emx
