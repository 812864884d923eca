/*
 * hkb_mpnn.h -- C ABI of the B200-native ProteinMPNN v_48_020 design engine.
 *
 * Drop-in for the design path of megure-labs/hikoboshi.  Each entry point
 * names the reference interface it replaces (paths relative to the reference
 * repository).  Plain pointers and sizes only; every input and output buffer
 * is caller-owned, the engine owns only its device memory.  No exceptions
 * cross this boundary and no call spawns threads.
 *
 * Status codes and the static, never-owned detail string follow
 * cpp/include/hikoboshi/universal/status.hpp:12-33.
 *
 * Shapes (B proteins, protein b has L_b residues and S_b sequences,
 * R = sum_b L_b, Q = sum_b S_b * L_b):
 *   coords        f32 [R, 5, 3]   canonical N, CA, C, O, CB slots
 *                                  (cpp/include/hikoboshi/universal/structure.hpp:21-38)
 *   atom_sources  u8  [R, 5]      0 Missing, 1 Observed, 2 Inferred, 3 Virtual
 *   tokens        i32 [Q]         alphabet "ACDEFGHIKLMNPQRSTVWYX"
 *   log_probs     f32 [Q, 21]
 *   orders        i32 [Q]         decoding order, residue index per position
 *   scores        f32 [sum_b S_b]  mean NLL over active residues
 * Protein b's sequences are contiguous; sequence s of protein b occupies
 * rows [qoff_b + s*L_b, qoff_b + (s+1)*L_b) of the [Q]-shaped arrays.
 */
#ifndef HKB_MPNN_H
#define HKB_MPNN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HKB_MPNN_ABI_VERSION 1

typedef enum {
  HKB_OK = 0,
  HKB_INVALID_ARGUMENT = 1,
  HKB_FAILED_PRECONDITION = 2,
  HKB_UNAVAILABLE = 3,
  HKB_UNIMPLEMENTED = 4,
  HKB_INTERNAL_ERROR = 5
} hkb_status_code;

typedef struct {
  int32_t code;       /* hkb_status_code */
  const char* detail; /* static string, never owned by the caller */
} hkb_status;

typedef enum {
  /* fp32 weights and activations on CUDA cores: the parity mode, within
   * 1e-4 of the reference's fp32 log-probs. */
  HKB_PRECISION_FP32 = 0,
  /* bf16 weights/activations on tcgen05 tensor cores, fp32 accumulation,
   * fp32 LayerNorm and softmax.  bf16's 8-bit mantissa holds log-probs to
   * within 6e-2 of the fp32 reference (measured <= 4.7e-2), not the 2e-2 of
   * the fp16 mode. */
  HKB_PRECISION_BF16 = 1,
  /* fp16 weights/activations on tcgen05 tensor cores (same tensor-core rate
   * as bf16, 8x finer rounding), fp32 accumulation, LayerNorm and softmax:
   * the throughput mode. */
  HKB_PRECISION_F16 = 2
} hkb_precision;

typedef enum {
  HKB_DECODE_RANDOM = 0, /* decode_order_scalar.cpp:89-116, seed + index */
  HKB_DECODE_N_TO_C = 1, /* identity order (algorithms/inverse_fold.cpp:273-276) */
  HKB_DECODE_INPUT = 2   /* caller permutation from input_orders */
} hkb_decode_order;

typedef struct hkb_engine hkb_engine;

typedef struct {
  int32_t num_proteins;
  const int32_t* residue_counts; /* [B] */
  const float* coords;           /* [R,5,3] host (or device for *_device) */
  const uint8_t* atom_sources;   /* [R,5]   host (or device for *_device) */
  const int32_t* num_seqs;       /* [B] sequences per protein, > 0 */
  const uint64_t* seeds;         /* [B] base seed; sequence s uses seed + s
                                    (algorithms/inverse_fold.cpp:186-189) */
  const float* temperatures;     /* [B] finite, >= 0; 0 = greedy */
  const int32_t* decode_orders;  /* [B] hkb_decode_order */
  const int32_t* input_orders;   /* [R] host; used where decode_order == INPUT */
} hkb_design_batch;

typedef struct {
  int32_t* tokens;  /* [Q] required */
  float* log_probs; /* [Q,21] optional (NULL = not returned) */
  int32_t* orders;  /* [Q] optional */
  float* scores;    /* [sum S] optional */
} hkb_design_out;

typedef struct {
  int32_t num_proteins;
  const int32_t* residue_counts; /* [B] */
  const float* coords;           /* [R,5,3] host */
  const uint8_t* atom_sources;   /* [R,5]   host */
  const int32_t* num_seqs;       /* [B] sequences scored per protein */
  const int32_t* tokens;         /* [Q] host, 0..20 */
  const int32_t* orders;         /* [Q] host permutations, or NULL: random
                                    order from seeds[b] + s */
  const uint64_t* seeds;         /* [B] used when orders == NULL */
} hkb_score_batch;

typedef struct {
  float* log_probs; /* [Q,21] unscaled log-softmax, required */
  int32_t* orders;  /* [Q] optional: the orders used */
  float* scores;    /* [sum S] optional */
} hkb_score_out;

/* Engine construction from the 118-tensor fp32 safetensors image (the
 * reference's embedded weights, weights/Hikoboshi-ProteinMPNN-v48-020
 * .safetensors, bound by name as cpp/weights/embedded_proteinmpnn_v48_eps020
 * .cpp:145-286 does).  Replaces embedded_proteinmpnn_v48_eps020_handle() +
 * make_prepared_weights() (cpp/weights/embedded_proteinmpnn_v48_eps020.cpp:
 * 276-331) and Engine construction (cpp/include/hikoboshi/api/engine.hpp:
 * 159-160).  One engine per device per host thread. */
hkb_status hkb_mpnn_create(const void* safetensors, size_t length, int device,
                           int32_t precision, hkb_engine** engine);

void hkb_mpnn_destroy(hkb_engine* engine);

/* Batched autoregressive design with host buffers; synchronous.  Replaces
 * the per-sequence loop of algorithms::inverse_fold_proteinmpnn_v48_020
 * (cpp/algorithms/inverse_fold.cpp:221-356) around
 * modules::mpnn::proteinmpnn_inverse_fold_scalar
 * (cpp/modules/mpnn/inverse_fold_scalar.cpp:954-1000), for many proteins at
 * once.  Validation mirrors algorithms/inverse_fold.cpp:232-261.
 * A log_probs buffer in page-locked, mapped host memory (cudaHostAlloc,
 * cudaHostRegister) is written by the 16-bit engines' decode kernel directly
 * as it samples, with no copy after the kernel; any other buffer receives a
 * copy.  The results are identical either way. */
hkb_status hkb_mpnn_design(hkb_engine* engine, const hkb_design_batch* batch,
                           hkb_design_out* out);

/* Same computation with coords / atom_sources already in device memory and
 * device output buffers, enqueued on `stream` (a cudaStream_t, NULL = the
 * engine's stream).  Host metadata (counts, seeds, temperatures, orders)
 * stays on the host.  Returns after enqueueing. */
hkb_status hkb_mpnn_design_device(hkb_engine* engine,
                                  const hkb_design_batch* batch,
                                  hkb_design_out* device_out, void* stream);

/* Teacher-forced scoring: one causally masked decoder pass per sequence.
 * Replaces modules::mpnn::proteinmpnn_teacher_forced_forward_scalar
 * (cpp/modules/mpnn/inverse_fold_scalar.cpp:905-952). */
hkb_status hkb_mpnn_score(hkb_engine* engine, const hkb_score_batch* batch,
                          hkb_score_out* out);

/* Encoder outputs for one protein: h_v f32 [L,128], h_e f32 [L,K,128],
 * e_idx i32 [L,K], K = min(48, L) (h_e in the engine precision, widened).
 * Exposes the intermediate of encode_backbone
 * (cpp/modules/mpnn/inverse_fold_scalar.cpp:300-352). */
hkb_status hkb_mpnn_encode(hkb_engine* engine, int32_t residue_count,
                           const float* coords, const uint8_t* atom_sources,
                           float* h_v, float* h_e, int32_t* e_idx);

/* CA top-K neighbour graph on the device, bit-exact with
 * primitives::compute::knn_scalar as build_knn configures it
 * (cpp/primitives/compute/knn_scalar.cpp:72-168,
 *  cpp/modules/mpnn/inverse_fold_scalar.cpp:211-234).  e_idx i32 [L,K],
 * d2 f32 [L,K] (optional). */
hkb_status hkb_mpnn_knn(hkb_engine* engine, int32_t residue_count,
                        const float* coords, const uint8_t* atom_sources,
                        int32_t* e_idx, float* d2);

/* Allocation-free design for small batches.  No counterpart in the
 * reference: it exists for callers that must not allocate device memory
 * while they run -- e.g. a plugin whose host application owns all GPU memory
 * through its own pool allocator, or a latency-bound loop that cannot take
 * cudaMalloc's implicit device synchronisation.  Same inputs and outputs as
 * hkb_mpnn_design_device (device coords / atom_sources, device tokens,
 * log_probs, orders and scores, all four required) and the same results as
 * that entry point on an fp32 engine, for batches of at most
 * HKB_NOALLOC_MAX_RESIDUES residues, HKB_NOALLOC_MAX_SEQUENCES sequences and
 * HKB_NOALLOC_MAX_ROWS designed residues (larger batches: InvalidArgument).
 * It calls no cudaMalloc / cudaFree: its scratch is one fixed device array of
 * about 18 MiB that every GPU loading this library holds until exit.  The
 * first call on a device looks that array's address up (one-time set-up) and
 * should come before any stream capture.  All calls share the array, so calls
 * whose GPU work overlaps race; the call returns after its work completes.
 * Always runs the fp32 pipeline. */
#define HKB_NOALLOC_MAX_RESIDUES 64
#define HKB_NOALLOC_MAX_SEQUENCES 64
#define HKB_NOALLOC_MAX_ROWS 1024
hkb_status hkb_mpnn_design_noalloc(hkb_engine* engine,
                                   const hkb_design_batch* batch,
                                   hkb_design_out* device_out, void* stream);

/* Host-only helpers (no device work) ----------------------------------- */

/* Decoding order, as proteinmpnn_decode_order_scalar
 * (cpp/modules/mpnn/decode_order_scalar.cpp:61-116): random from `seed`
 * (residue_mask may be NULL = all ones) or a validated caller permutation. */
hkb_status hkb_mpnn_decode_order(int32_t residue_count, const float* residue_mask,
                                 uint64_t seed, int32_t decode_order,
                                 const int32_t* input_order, int32_t* order);

/* Seeded synthetic single-chain backbone (benchmark input generator; no
 * counterpart in the reference).  Ideal N-CA-C-O geometry, runs of helix /
 * strand phi/psi, virtual CB.  coords f32 [L,5,3], sources u8 [L,5]. */
hkb_status hkb_synthetic_backbone(uint64_t seed, int32_t residue_count,
                                  float* coords, uint8_t* atom_sources);

/* Number of tcgen05/CUDA kernel launches the last design/score call made. */
int64_t hkb_mpnn_last_launch_count(const hkb_engine* engine);

/* Device milliseconds of the last call's phases: [0] featurise+encode,
 * [1] decoder preparation, [2] decode / score, [3] total. */
hkb_status hkb_mpnn_last_timings(const hkb_engine* engine, float* ms4);

int32_t hkb_mpnn_abi_version(void);

/* ---- host-side input / output of the design command (no device work) ---- */

/* A structure loaded from PDB or mmCIF: one chain of one model, normalised to
 * the canonical [L,5,3] N/CA/C/O/CB layout with per-atom sources
 * (0 missing, 1 observed, 2 inferred, 3 virtual).
 * Replaces io::LoadedStructure / io::load_structure_from_file
 * (cpp/include/hikoboshi/io/structure_loader.hpp; io/structure_loader.cpp:174-284). */
typedef struct hkb_structure hkb_structure;

/* io::StructureLoadOptions (structure_loader.hpp:30-38); NULL = defaults. */
typedef struct {
  int32_t model_index;               /* 0: model 1 */
  const char* chain_id;              /* NULL or "": chain A if present, else the first */
  int32_t infer_missing_atoms;       /* default 1 */
  int32_t include_modified_residues; /* default 1 (MSE, SEC, PYL, SEP, TPO, PTR, HYP) */
} hkb_structure_options;

/* Reads a .pdb/.ent/.cif/.mmcif file (format by extension, then content).
 * Errors carry the reference's codes and detail strings. */
hkb_status hkb_structure_load_file(const char* path, const hkb_structure_options* options,
                                   hkb_structure** out);
/* Same from text; format 0 = detect from content, 1 = PDB, 2 = mmCIF
 * (io::load_pdb_from_string / load_mmcif_from_string, structure_loader.cpp:202-284). */
hkb_status hkb_structure_load_text(const char* text, size_t length, int32_t format,
                                   const char* origin, const hkb_structure_options* options,
                                   hkb_structure** out);
int32_t hkb_structure_residue_count(const hkb_structure* structure);
/* coords f32 [L,5,3], atom_sources u8 [L,5], residue_codes char [L] (any may be NULL). */
hkb_status hkb_structure_copy(const hkb_structure* structure, float* coords,
                              uint8_t* atom_sources, char* residue_codes);
void hkb_structure_destroy(hkb_structure* structure);

/* Backbone noise of one sequence (algorithms/inverse_fold.cpp:191-207): out =
 * coords + N(0, sigma) on every non-missing atom, drawn x, y, z per atom from
 * std::mt19937_64(seed ^ 0x4D504E4E76343875) through
 * std::normal_distribution<float> -- the host's libstdc++, as the reference.
 * seed is the sequence's seed (base + index); sigma must be finite and >= 0. */
hkb_status hkb_backbone_noise(int32_t residue_count, const float* coords,
                              const uint8_t* atom_sources, float sigma, uint64_t seed,
                              float* out);

/* Design FASTA (io::write_design_fasta, io/design_fasta_writer.cpp:171-199):
 * ">design_<i> score=<score> seed=<seed> T=<T> decode_order=<random|n_to_c>",
 * sequences wrapped at 80 columns.  tokens i32 [num_seqs, L]. */
hkb_status hkb_write_design_fasta(const char* path, int32_t num_seqs, int32_t residue_count,
                                  const int32_t* tokens, const double* scores,
                                  const uint64_t* seeds, float sampling_temp,
                                  int32_t decode_order);

/* Log-prob NPZ (io::write_inverse_fold_logprobs_npz, :201-217): one stored
 * (uncompressed) ZIP32 member log_probs.npy, float32 [num_seqs, L, 21]. */
hkb_status hkb_write_logprobs_npz(const char* path, int32_t num_seqs, int32_t residue_count,
                                  const float* log_probs);

#ifdef __cplusplus
}
#endif
#endif /* HKB_MPNN_H */
