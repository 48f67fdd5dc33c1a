// step.cu — planning and cooperative launch of the persistent token-step kernel (step.cuh).
#include <algorithm>
#include <string>
#include <vector>

#include "host.h"
#include "step.cuh"

namespace fence {

struct StepPlan {
    int ok = 0;
    int grid = 0, block = SK_NT, smem = 0;
    int ring = 0, slot_bytes = 0, scratch_bytes = 0, acc_floats = 0;
};

// Geometry of one GEMV phase for SK_NL consumer lanes (stages of R actual rows).
static bool plan_step_gemv(RGemvArgs& g, int grid, std::string& err) {
    const int I = g.I;
    if (I <= 0 || g.Mv <= 0) {
        err = "step kernel: empty GEMV phase";
        return false;
    }
    const int vcta = (g.Mv + grid - 1) / grid;
    const int rows_cta = vcta * (g.dual ? 2 : 1);
    // tiles of RB rows x CI items, one item per consumer lane: slices of 8 to 32 items (a row's lanes
    // inside one warp), as many rows of the CTA per block as the lanes allow
    const int CI = std::max(1, std::min(std::min(I, 32), std::max(8, SK_NL / std::max(1, rows_cta))));
    const int RB = std::max(1, std::min(rows_cta, SK_NL / CI));
    int mp = 1;
    for (int r = 0; r < RB; ++r) mp = std::max(mp, rg_part_pieces(r, 0, 1, CI));
    g.np = 1;
    g.ipl = 1;
    g.R = RB;
    g.RB = RB;
    g.CI = CI;
    g.mp = mp;
    g.rows_cta = rows_cta;
    g.ring = 0;
    g.slot_bytes = (int)((sk_tile_bytes(g.wt, RB, std::min(CI, I), CI) + 127u) & ~127u);
    return true;
}

static StepPlan plan_step(std::vector<SPhase>& phases, int dev, std::string& err) {
    StepPlan P;
    int sms = 0, optin = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int grid = sms;
    int scratch = sk_attn_scratch_bytes();
    int slot = 0, accf = 0;
    for (SPhase& ph : phases) {
        if (ph.kind != SP_GEMV) continue;
        if (!plan_step_gemv(ph.g, grid, err)) return P;
        slot = std::max(slot, ph.g.slot_bytes);
        accf = std::max(accf, ph.g.rows_cta * ph.g.mp);
        int need = ph.g.I * (int)SK_XQB;
        if (ph.embed || ph.tp_sum) need += ph.g.I * 64 * 4;  // fp32 x row (embedding / reduced) after the records
        scratch = std::max(scratch, need);
        if (ph.moe) accf = std::max(accf, SK_NW * SK_MOE_EMAX);  // the router's reduction (sk_route)
    }
    P.scratch_bytes = (scratch + 15) / 16 * 16;
    P.acc_floats = accf;
    P.slot_bytes = slot;
    int ring = 8;
    while (ring > 2 && (int)sk_smem_layout(ring, slot, P.scratch_bytes, accf).total > optin) --ring;
    if ((int)sk_smem_layout(ring, slot, P.scratch_bytes, accf).total > optin) {
        err = "step kernel: the shared-memory plan does not fit";
        return P;
    }
    P.ring = ring;
    P.smem = (int)sk_smem_layout(ring, slot, P.scratch_bytes, accf).total;
    P.grid = grid;
    P.ok = 1;
    return P;
}

template <typename KVT, bool TP>
static cudaError_t launch_step_k(const StepArgs& a, const StepPlan& P, cudaStream_t st) {
    auto kern = step_kernel<KVT, TP>;
    static int smem_set[64] = {};  // per device: largest dynamic smem enabled so far
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem_set[dev] < P.smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P.smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, P.block, P.smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
        smem_set[dev] = P.smem;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.grid);
    cfg.blockDim = dim3(P.block);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the phase counter needs it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename KVT>
static cudaError_t launch_step(const StepArgs& a, const StepPlan& P, cudaStream_t st) {
    return a.tp_n > 1 ? launch_step_k<KVT, true>(a, P, st) : launch_step_k<KVT, false>(a, P, st);
}

}  // namespace fence
