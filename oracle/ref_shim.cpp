// C entry points over the reference's own CPU reference (harness/k3/ref.h of
// the reference project, compiled from where it lies; nothing is copied).
// TEST INFRASTRUCTURE ONLY: tests/golden/make_golden.py runs it here to make
// golden vectors; the GPU box never needs it.
#include "ref.h"

extern "C" {
int k3ref_experts(void) { return k3ref::EXPERTS; }
int k3ref_topk(void) { return k3ref::TOPK; }
// ref_router_topk: S f32 [B, 896], bias f32 [896], rs bf16 [1] -> idx [B, 16], wts [B, 16]
void k3ref_router_topk(const float* S, const float* bias, const uint16_t* rs, int* idx, float* wts, int B) {
  k3ref::ref_router_topk(S, bias, rs, idx, wts, B);
}
// ref_land_situ: p f32 [B, 2n] (gate | up) -> act bf16 [B, n], K3's SiTU with bf16 landings
void k3ref_land_situ(const float* p, uint16_t* act, int n, int B) {
  k3ref::ref_land_situ(p, act, n, B);
}
}
