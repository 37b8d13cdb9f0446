// The exported launcher tables (crates/pc-kernels/kernels/args.cuh:1034-1119): the reference's L3 seam.
// Entries outside this library's hot path are non-null and return -1 ("argument out of the kernel's range"), as the
// reference's own tables do for kernels an instantiation lacks.
#include "kernels.h"

namespace {
int absent(const void*, cudaStream_t) { return -1; }
// the reference's small_int is defined for 32-bit words only; its 64-bit tables answer -2 (crates/pc-kernels/kernels/bts.cuh)
int words32_only(const void*, cudaStream_t) { return -2; }

template <int LOGN>
PcbKernelTable make_table() {
    using namespace pcb;
    PcbKernelTable t;
    PcbLaunch* all = (PcbLaunch*)&t.ntt_fwd;
    for (int i = 0; i < 52; ++i) all[i] = absent;
    t.abi = PCB_KERNELS_ABI;
    t.word_bytes = 8;
    t.mm = 0;
    t.log_n = LOGN;
    t.ntt_fwd = ntt::fwd<LOGN>;
    t.ntt_inv = ntt::inv<LOGN>;
    t.bconv = ks::bconv_launch<LOGN>;
    // on 64-bit words the reference's wide conversion takes the same jobs (up to 16 sources) with the same sums
    t.bconv_wide = ks::bconv_launch<LOGN>;
    t.ew_add = elem::ew_launch<LOGN, elem::ADD>;
    t.ew_scale = elem::ew_launch<LOGN, elem::SCALE>;
    t.ew_sub_mul = elem::ew_launch<LOGN, elem::SUB_MUL>;
    t.ew_copy = elem::ew_launch<LOGN, elem::COPY>;
    t.ks_dot = ks::ks_dot_launch<LOGN>;
    t.ks_dot_regen = regen::ks_dot_regen_launch<LOGN>;
    t.ks_dot_key = regen::ks_dot_key_launch<LOGN>;
    t.cts_fused = cts::cts_fused_launch<LOGN>;
    t.cts_fused_regen = cts::cts_fused_regen_launch<LOGN>;
    t.ksk_expand = keys::ksk_expand_launch<LOGN>;
    t.pt_dot = pt::pt_dot_launch<LOGN>;
    t.coeff_sum = pt::coeff_sum_launch<LOGN>;
    t.add_const = pt::add_const_launch<LOGN>;
    t.mul_table = pt::mul_table_launch<LOGN>;
    t.mul_add = pt::mul_add_launch<LOGN>;
    t.mul_add_n = pt::mul_add_n_launch<LOGN>;
    t.tensor = elem::tensor_launch<LOGN>;
    t.tensor_y = elem::tensor_y_launch<LOGN>;
    t.md_epilogue = elem::md_epilogue_launch<LOGN>;
    t.rescale_coef = elem::rescale_coef_launch<LOGN>;
    t.rescale_combine = elem::rescale_combine_launch<LOGN>;
    t.automorph = elem::automorph_launch<LOGN>;
    t.encrypt = keys::encrypt_launch<LOGN>;
    t.ksk_gen = keys::ksk_gen_launch<LOGN>;
    t.ksk_unpack = keys::ksk_unpack_launch<LOGN>;
    t.mod_raise = elem::mod_raise_launch<LOGN>;
    t.small_int1 = elem::small_int1_launch<LOGN>;
    t.small_int = words32_only;
    t.wsum = elem::wsum_launch<LOGN>;
    t.wsum_k = elem::wsum_k_launch<LOGN>;
    t.wsum_multi = elem::wsum_multi_launch<LOGN>;
    t.rescale_combine_to = elem::rescale_combine_to_launch<LOGN>;
    t.rescale_fwd = elem::rescale_fwd_launch<LOGN>;
    t.md_epilogue_to = elem::md_epilogue_to_launch<LOGN>;
    t.tensor_sum = elem::tensor_sum_launch<LOGN>;
    t.tensor_multi = elem::tensor_multi_launch<LOGN>;
    t.ew_many = elem::ew_many_launch<LOGN>;
    t.submul_many = elem::submul_many_launch<LOGN>;
    t.pack_split = elem::pack_split_launch<LOGN>;
    t.pack_dot = elem::pack_dot_launch<LOGN>;
    return t;
}

template <int LOGN>
PcbRingTable make_ring() {
    using namespace pcb;
    PcbRingTable r;
    r.abi = PCB_RING_ABI;
    r.word_bytes = 8;
    r.mm = 0;
    r.log_n = LOGN;
    r.ntt_fwd = ntt::fwd<LOGN>;
    r.ntt_inv = ntt::inv<LOGN>;
    r.ntt_fwd_g = ntt::fwd<LOGN>;
    r.ntt_inv_g = ntt::inv<LOGN>;
    r.bconv = ks::bconv_launch<LOGN>;
    r.ew_add = elem::ew_launch<LOGN, elem::ADD>;
    r.ew_scale = elem::ew_launch<LOGN, elem::SCALE>;
    r.ew_sub_mul = elem::ew_launch<LOGN, elem::SUB_MUL>;
    r.ew_copy = elem::ew_launch<LOGN, elem::COPY>;
    return r;
}

const PcbKernelTable g_table16 = make_table<16>();
const PcbKernelTable g_table14 = make_table<14>();
const PcbRingTable g_ring14 = make_ring<14>();
const PcbRingTable g_ring16 = make_ring<16>();
}  // namespace

#include <atomic>

namespace {
std::atomic<unsigned long long> g_launches{0};
}

namespace pcb {
void note_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// the full launcher set at either ring size, for the evaluator
const PcbKernelTable* table_for(int logn) { return logn == 14 ? &g_table14 : logn == 16 ? &g_table16 : nullptr; }
}  // namespace pcb

extern "C" {
uint64_t pcb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }
const PcbKernelTable* pc_table_u64_barrett64(void) { return &g_table16; }
const PcbRingTable* pc_ring_u64_14(void) { return &g_ring14; }
const PcbRingTable* pc_ring_u64_16(void) { return &g_ring16; }
const PcbKernelTable* pcb_kernel_table(int32_t log_n) { return pcb::table_for(log_n); }
}
