// Binary launch-plan format shared by the plan emitter (emx_onnx_cgen_b200/plan.py,
// which packs these records with `struct`) and the runtime (runtime.cu).
//
// Layout (little-endian, every record 8-byte aligned):
//   PlanHeader
//   PlanTensor[n_tensors]
//   uint32_t input_tensor_ids[n_inputs]   (padded to a multiple of 2 entries)
//   uint32_t output_tensor_ids[n_outputs] (padded to a multiple of 2 entries)
//   PlanOp[n_ops]                          (execution order = LoweredModel.ops order)
//
// The plan replaces the generated C's static storage decisions: every tensor
// has a fixed offset either in the weight blob or in one device arena sized at
// emit time, so nothing is allocated while running (the generated C instead
// malloc's large temporaries per call, reference c_emitter.py:2744-2789).
#pragma once
#include <stdint.h>

#define EMX_PLAN_MAGIC 0x50584D45u  // "EMXP"
#define EMX_PLAN_VERSION 1u
#define EMX_MAX_RANK 8
#define EMX_OP_MAX_TENSORS 12
#define EMX_OP_MAX_IPARAMS 40
#define EMX_OP_MAX_FPARAMS 8

enum EmxTensorKind : uint32_t {
  EMX_T_WEIGHT = 0,  // offset into the weight blob
  EMX_T_INPUT = 1,   // graph input; offset = host-staging slot in the arena
  EMX_T_OUTPUT = 2,  // graph output; offset = host-staging slot in the arena
  EMX_T_TEMP = 3,    // intermediate; offset into the arena
};

enum EmxDtype : uint32_t {
  EMX_F32 = 1, EMX_U8 = 2, EMX_I8 = 3, EMX_I32 = 6, EMX_I64 = 7, EMX_F16 = 10, EMX_F64 = 11,
};

enum EmxPlanFlags : uint32_t {
  EMX_PLAN_BATCHABLE = 1u,  // every batched I/O tensor has batch_axis 0: run() may slice
};

struct PlanHeader {
  uint32_t magic, version;
  uint32_t n_tensors, n_ops, n_inputs, n_outputs;
  int64_t batch;          // full batch along axis 0 of batched I/O (0 = none)
  uint64_t arena_bytes;   // device arena (temps + I/O staging + error word)
  uint64_t weight_bytes;  // size of the weight blob
  uint32_t flags, reserved;
};
static_assert(sizeof(PlanHeader) == 56, "PlanHeader layout");

struct PlanTensor {
  uint32_t kind, dtype;
  uint64_t offset, nbytes;
  int32_t rank, batch_axis;  // batch_axis -1: not sliced by run()
  int64_t dims[EMX_MAX_RANK];
};
static_assert(sizeof(PlanTensor) == 96, "PlanTensor layout");

struct PlanOp {
  uint32_t kernel, n_tensors;
  int32_t t[EMX_OP_MAX_TENSORS];   // tensor ids (-1 = absent)
  int64_t ip[EMX_OP_MAX_IPARAMS];  // kernel-specific integers (kernels.h)
  double fp[EMX_OP_MAX_FPARAMS];   // kernel-specific reals
};
static_assert(sizeof(PlanOp) == 440, "PlanOp layout");
