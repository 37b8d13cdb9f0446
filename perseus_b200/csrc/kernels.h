// Internal declarations of the launchers (one instantiation per ring size LOGN in {14, 16}).
#pragma once
#include "../../include/pcb200.h"

namespace pcb {
namespace ntt {
template <int LOGN> int fwd(const PcbNttArgs*, cudaStream_t);
template <int LOGN> int inv(const PcbNttArgs*, cudaStream_t);
// f64: every prime of the launch is below 2^50 and fw/fws (iw/iws) hold centred double twiddles w and fl(w / p)
template <int LOGN> int fwd_run(const PcbNttArgs*, bool f64, cudaStream_t);
template <int LOGN> int inv_run(const PcbNttArgs*, bool f64, cudaStream_t);
}  // namespace ntt
namespace elem {
enum EwOpDecl { ADD = 0, SCALE = 1, SUB_MUL = 2, COPY = 3 };
// out = sum of n batches of ciphertexts mod p, rows 0 .. nrows-1 of both parts (an internal launch, not a table entry)
constexpr int SUM_MAX = 32;
struct SumArgs {
    const uint64_t* in[SUM_MAX];
    uint64_t* out;
    const PcbPrimeConst* pr;
    uint64_t ct_stride, part_stride;  // words
    int32_t n, nrows, K;
};
template <int LOGN> int sum_launch(const SumArgs*, cudaStream_t);
template <int LOGN, int OP> int ew_launch(const PcbEwArgs*, cudaStream_t);
template <int LOGN> int tensor_launch(const PcbTensorArgs*, cudaStream_t);
template <int LOGN> int tensor_y_launch(const PcbTensorYArgs*, cudaStream_t);
template <int LOGN> int md_epilogue_launch(const PcbMdEpiArgs*, cudaStream_t);
template <int LOGN> int rescale_coef_launch(const PcbRescaleArgs*, cudaStream_t);
template <int LOGN> int rescale_combine_launch(const PcbRescaleCombineArgs*, cudaStream_t);
template <int LOGN> int mod_raise_launch(const PcbModRaiseArgs*, cudaStream_t);
template <int LOGN> int small_int1_launch(const PcbSmallInt1Args*, cudaStream_t);
template <int LOGN> int automorph_launch(const PcbAutomorphArgs*, cudaStream_t);
}  // namespace elem
namespace pt {
template <int LOGN> int add_const_launch(const PcbAddConstArgs*, cudaStream_t);
template <int LOGN> int mul_table_launch(const PcbMulTableArgs*, cudaStream_t);
template <int LOGN> int mul_add_launch(const PcbMulAddArgs*, cudaStream_t);
template <int LOGN> int mul_add_n_launch(const PcbMulAddNArgs*, cudaStream_t);
template <int LOGN> int pt_dot_launch(const PcbPtDotArgs*, cudaStream_t);
template <int LOGN> int coeff_sum_launch(const PcbCoeffArgs*, cudaStream_t);
}  // namespace pt
namespace ks {
template <int LOGN> int bconv_launch(const PcbBconvArgs*, cudaStream_t);
template <int LOGN> int ks_dot_launch(const PcbKsArgs*, cudaStream_t);
// narrow = every residue and constant of the launch is below 2^52 (26-bit-split accumulators; ks_dot: K <= 4)
// ns_all: the source count shared by every job of the launch (0: mixed)
// f64: every prime of the launch below 2^50 (FP64 products)
template <int LOGN> int bconv_run(const PcbBconvArgs*, bool narrow, bool f64, int ns_all, cudaStream_t);
template <int LOGN> int ks_dot_run(const PcbKsArgs*, bool narrow, cudaStream_t);
// Up to KEYS_MAX keys against the same inputs in one launch (hoisted rotations): key pointers and automorphism
// indices by value; key r's outputs go to out0 / out1 + r out_rot_stride. FP64 form (every prime below 2^50).
// Key r's `a` is read from ka[r] (dense) or regenerated from the 8-word device seed seed[r] (keyregen.cuh); every key
// of one launch has the same source.
constexpr int KEYS_MAX = 4;
struct KeyGroup {
    const uint64_t* kb[KEYS_MAX];
    const uint64_t* ka[KEYS_MAX];
    const uint32_t* seed[KEYS_MAX];
    uint32_t autok[KEYS_MAX];
    int32_t n;
};
template <int LOGN> int dot_keys_run(const PcbKsArgs*, const KeyGroup&, cudaStream_t);
// The keys of a rotate_sum group summed into ONE extended batch (out0 / out1, out_ct_stride), gather form: g[r] is
// key r's Galois element (its output slot o reads slot automorph_slot(g[r], o)). FP64 form (every prime below 2^50);
// c0_mode 0 or 1, optionally | PCB_KS_ACC.
constexpr int SUM_KEYS_MAX = 8;
struct KeySum {
    const uint64_t* kb[SUM_KEYS_MAX];
    const uint64_t* ka[SUM_KEYS_MAX];
    const uint32_t* seed[SUM_KEYS_MAX];  // as KeyGroup

    uint32_t g[SUM_KEYS_MAX];
    int32_t n;
};
template <int LOGN> int dot_sum_run(const PcbKsArgs*, const KeySum&, cudaStream_t);
// one key, any batch K: key words read once per launch; inputs must not alias outputs
// f64: every prime below 2^50 (FP64 products); seed non-null: the key's `a` is regenerated from that 8-word device
// seed (keyregen.cuh) and a.ka is not read
template <int LOGN> int dot_all_run(const PcbKsArgs*, bool narrow, bool f64, const uint32_t* seed, cudaStream_t);
}  // namespace ks
namespace regen {
template <int LOGN> int ks_dot_regen_launch(const PcbKsRegenArgs*, cudaStream_t);
template <int LOGN> int ks_dot_key_launch(const PcbKsKeyArgs*, cudaStream_t);
}  // namespace regen
namespace cts {
template <int LOGN> int cts_fused_launch(const PcbCtsArgs*, cudaStream_t);
template <int LOGN> int cts_fused_regen_launch(const PcbCtsRegenArgs*, cudaStream_t);
}  // namespace cts
namespace elem {  // elem_multi.cu
template <int LOGN> int ew_many_launch(const PcbEwManyArgs*, cudaStream_t);
template <int LOGN> int submul_many_launch(const PcbSubMulManyArgs*, cudaStream_t);
template <int LOGN> int pack_split_launch(const PcbPackSplitArgs*, cudaStream_t);
template <int LOGN> int pack_dot_launch(const PcbPackDotArgs*, cudaStream_t);
template <int LOGN> int wsum_launch(const PcbWsumArgs*, cudaStream_t);
template <int LOGN> int wsum_k_launch(const PcbWsumKArgs*, cudaStream_t);
template <int LOGN> int wsum_multi_launch(const PcbWsumMultiArgs*, cudaStream_t);
template <int LOGN> int tensor_sum_launch(const PcbTensorSumArgs*, cudaStream_t);
template <int LOGN> int tensor_multi_launch(const PcbTensorMultiArgs*, cudaStream_t);
template <int LOGN> int md_epilogue_to_launch(const PcbMdEpiToArgs*, cudaStream_t);
template <int LOGN> int rescale_combine_to_launch(const PcbRescaleCombineToArgs*, cudaStream_t);
template <int LOGN> int rescale_fwd_launch(const PcbRescaleNttArgs*, cudaStream_t);
}  // namespace elem
namespace keys {
template <int LOGN> int ksk_expand_launch(const PcbKskExpandArgs*, cudaStream_t);
template <int LOGN> int encrypt_launch(const PcbEncryptArgs*, cudaStream_t);
template <int LOGN> int ksk_gen_launch(const PcbKskGenArgs*, cudaStream_t);
template <int LOGN> int ksk_unpack_launch(const PcbKskUnpackArgs*, cudaStream_t);
}  // namespace keys
// wire.cu: the compressed ciphertext frame of k <= 2 coefficient rows per part (both parts), `bits` per coefficient
int wire_compress_launch(const uint64_t* coef, int k, size_t n, const PcbPrimeConst& c0, const PcbPrimeConst& c1,
                         uint64_t inv01, int bits, uint32_t* out, cudaStream_t s);
}  // namespace pcb
