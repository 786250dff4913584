// Torch-facing wrappers of the tcgen05 flash-attention forward and backward kernels.
#include "common.cuh"

extern "C" int vo_fmha_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                           int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_error(int reset);
extern "C" int vo_fmha_fwd2(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            int B, int H, int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_fwd2_error(int reset);
extern "C" int vo_fmha_fwd3(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            int B, int H, int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_fwd3_kvlen(const void* q, const void* k, const void* v, void* o, void* o2, int out_split,
                                  float* lse, const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale,
                                  cudaStream_t stream);
extern "C" int vo_fmha_fwd_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                int H, int Sq, int Skv, int D, float scale, cudaStream_t stream);
extern "C" int vo_fmha_fwd4(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                            cudaStream_t stream);
extern "C" int vo_fmha_fwd4_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                 void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                 int H, int Sq, int Skv, int D, float scale, cudaStream_t stream);
extern "C" int vo_fmha_fwd5(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                            cudaStream_t stream);
extern "C" int vo_fmha_fwd5_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                 void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                 int H, int Sq, int Skv, int D, float scale, cudaStream_t stream);
extern "C" int vo_fmha_fwd4v(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                             const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                             cudaStream_t stream, int variant);
extern "C" int vo_fmha_bwd_trace(long long* host);
extern "C" int vo_fmha_bwd(const void* q, const void* k, const void* v, const void* o, const void* dO,
                           const void* o2, const void* dO2, int split, const float* lse, void* dq, void* dk, void* dv,
                           float* delta, float* dq_acc, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                           cudaStream_t stream, int version, const int* kv_len);
extern "C" int vo_fmha_bwd_error(int reset);

namespace vo {

// q [B, H, Sq, D], k/v [B, H, Skv, D] -> (o [B, Sq, H, D], lse [B, H, Sq] fp32[, o2])
// version 1: one query tile per CTA, P staged in shared memory; version 2: two query tiles per CTA,
// P and O resident in tensor memory; version 3: as 2 with two softmax warpgroups per query tile;
// version 4: one query tile per CTA, two CTAs per SM, double-buffered 64-key score blocks (key counts
// and the causal mask both supported); version 5: as 4 with two independent softmax halves per tile at
// head_dim 64 (other widths run version 4).
// split > 0 (versions 2 / 3): query rows [0, split) go to o [B, split, H, D] and rows [split, Sq) to a
// second tensor o2 [B, Sq - split, H, D] (the image / text halves of a joint attention, each feeding
// its own output projection without a copy).
std::vector<torch::Tensor> fmha_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale,
                                    int64_t version, int64_t split, c10::optional<torch::Tensor> kv_len) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "bf16 attention inputs");
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(split >= 0 && split < Sq, "bad output split");
  TORCH_CHECK(split == 0 || version >= 2, "split outputs need forward version 2, 3 or 4");
  auto o = torch::empty({B, split > 0 ? split : Sq, H, D}, q.options());
  torch::Tensor o2 = split > 0 ? torch::empty({B, Sq - split, H, D}, q.options()) : torch::Tensor();
  auto lse = torch::empty({B, H, Sq}, q.options().dtype(torch::kFloat32));
  int rc;
  if (version >= 4) {
    const int* kvp = nullptr;
    if (kv_len.has_value() && kv_len->defined()) {
      VO_CHECK_INPUT((*kv_len));
      TORCH_CHECK(kv_len->scalar_type() == torch::kInt32 && kv_len->numel() == B, "int32 [B] key counts");
      kvp = kv_len->data_ptr<int>();
    }
    if (version >= 40) {  // version 4 with an explicit exponential split (measurements)
      rc = vo_fmha_fwd4v(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), split > 0 ? o2.data_ptr() : nullptr,
                         (int)split, lse.data_ptr<float>(), kvp, B, H, Sq, Skv, D, (float)scale, causal ? 1 : 0,
                         stream(), (int)version);
    } else {
      auto fn = version >= 5 ? vo_fmha_fwd5 : vo_fmha_fwd4;
      rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), split > 0 ? o2.data_ptr() : nullptr, (int)split,
              lse.data_ptr<float>(), kvp, B, H, Sq, Skv, D, (float)scale, causal ? 1 : 0, stream());
    }
  } else if (kv_len.has_value() && kv_len->defined()) {
    // per-sequence key counts (right-padded keys masked); non-causal, forward v3
    VO_CHECK_INPUT((*kv_len));
    TORCH_CHECK(kv_len->scalar_type() == torch::kInt32 && kv_len->numel() == B && !causal, "int32 [B] key counts");
    rc = vo_fmha_fwd3_kvlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), split > 0 ? o2.data_ptr() : nullptr,
                            (int)split, lse.data_ptr<float>(), kv_len->data_ptr<int>(), B, H, Sq, Skv, D, (float)scale,
                            stream());
  } else if (version >= 2) {
    auto fn = version == 3 ? vo_fmha_fwd3 : vo_fmha_fwd2;
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), split > 0 ? o2.data_ptr() : nullptr, (int)split,
            lse.data_ptr<float>(), B, H, Sq, Skv, D, (float)scale, causal ? 1 : 0, stream());
  } else {
    rc = vo_fmha_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), B, H, Sq, Skv, D,
                     (float)scale, causal ? 1 : 0, stream());
  }
  TORCH_CHECK(rc == 0, "tcgen05 FMHA launch failed: code ", rc);
  count_launch();
  if (split > 0) return {o, lse, o2};
  return {o, lse};
}

// Ulysses attention with the output exchange fused into the epilogue (inference): q/k/v [B, H, Sq, D] hold
// this rank's H heads of the sequence gathered from the group (sl rows per rank: si image rows, then text);
// each output row is stored into the owning rank's buffer: peer_o[r] [B, si, htot, D] (image rows) or
// peer_o2[r] [B, sl - si, htot, D] (text rows), this rank's heads at head offset h0.
void fmha_fwd_peer(torch::Tensor q, torch::Tensor k, torch::Tensor v, std::vector<int64_t> peer_o,
                   std::vector<int64_t> peer_o2, int64_t sl, int64_t si, int64_t htot, int64_t h0, double scale,
                   int64_t version) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "bf16 attention inputs");
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  const int n = (int)peer_o.size();
  TORCH_CHECK(n >= 1 && n <= 8 && (peer_o2.empty() || (int)peer_o2.size() == n), "1..8 peer buffers");
  std::vector<void*> po(n), po2(n, nullptr);
  for (int i = 0; i < n; ++i) {
    po[i] = reinterpret_cast<void*>(peer_o[i]);
    if (!peer_o2.empty()) po2[i] = reinterpret_cast<void*>(peer_o2[i]);
  }
  auto lse = torch::empty({B, H, Sq}, q.options().dtype(torch::kFloat32));
  auto fn = version >= 5 ? vo_fmha_fwd5_peer : version == 4 ? vo_fmha_fwd4_peer : vo_fmha_fwd_peer;
  const int rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), po.data(), po2.data(), n, (int)sl, (int)si, (int)htot,
                    (int)h0, lse.data_ptr<float>(), B, H, Sq, Skv, D, (float)scale, stream());
  TORCH_CHECK(rc == 0, "tcgen05 FMHA (peer output) launch failed: code ", rc);
  count_launch();
}

int64_t fmha_error(bool reset) {
  return vo_fmha_error(reset ? 1 : 0) | vo_fmha_fwd2_error(reset ? 1 : 0) | vo_fmha_bwd_error(reset ? 1 : 0);
}

// returns dq, dk, dv in the [B, H, S, D] layout of q, k, v
// version 1: one key tile per CTA, serial per query tile; version 2: pipelined (P^T / dS^T in
// tensor memory, two gradient warpgroups, concurrent dQ drain).  split > 0: O and dO are given as
// two halves (o, dO: rows [0, split); o2, dO2: rows [split, Sq)); split must be a multiple of 128.
std::vector<torch::Tensor> fmha_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor lse, torch::Tensor dO, bool causal, double scale, int64_t version,
                                    c10::optional<torch::Tensor> o2, c10::optional<torch::Tensor> dO2, int64_t split,
                                    c10::optional<torch::Tensor> kv_len) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  VO_CHECK_INPUT(o);
  VO_CHECK_INPUT(dO);
  VO_CHECK_INPUT(lse);
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  const void* po2 = nullptr;
  const void* pdo2 = nullptr;
  if (split > 0) {
    TORCH_CHECK(split % 128 == 0 && split < Sq, "split must be a multiple of 128 below Sq");
    TORCH_CHECK(o2.has_value() && dO2.has_value(), "split needs o2 and dO2");
    VO_CHECK_INPUT((*o2));
    VO_CHECK_INPUT((*dO2));
    po2 = o2->data_ptr();
    pdo2 = dO2->data_ptr();
  }
  const int* kvp = nullptr;
  if (kv_len.has_value() && kv_len->defined()) {
    VO_CHECK_INPUT((*kv_len));
    TORCH_CHECK(kv_len->scalar_type() == torch::kInt32 && kv_len->numel() == B && !causal, "int32 [B] key counts");
    kvp = kv_len->data_ptr<int>();
  }
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  auto fo = q.options().dtype(torch::kFloat32);
  // Delta [B, H, Sq], then (16-byte aligned) the per-64-query-block lse / Delta records of version 4
  auto delta = torch::empty({B * H * Sq + B * H * ((Sq + 63) / 64) * 128 + 4}, fo);
  auto dq_acc = torch::zeros({B, H, Sq, D}, fo);
  int rc = vo_fmha_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dO.data_ptr(), po2, pdo2, (int)split,
                       lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr<float>(),
                       dq_acc.data_ptr<float>(), B, H, Sq, Skv, D, (float)scale, causal ? 1 : 0, stream(),
                       (int)version, kvp);
  TORCH_CHECK(rc == 0, "tcgen05 FMHA backward launch failed: code ", rc);
  count_launch(version >= 4 && version <= 8 ? 4 : 3);
  return {dq, dk, dv};
}

// Event stamps of the last traced backward launch (version 6): int64 [32 CTAs, 64 blocks, 16 slots] of
// SM clocks (0 = not reached).  Events: 0 Q/dO load issued, 1 MMA sees dS ready, 2 dV/dK/dQ issued,
// 3 next S/dP inputs ready, 4 gradient block start, 5 dS slots free, 6 S/dP ready, 7 dS written,
// 8 dQ ready at the drain, 9 dQ drained, 10 scores loaded from tensor memory, 11 exp / dS math done,
// 12 tensor-memory and shared stores issued, 13 tensor-memory stores complete.
torch::Tensor fmha_bwd_trace() {
  auto out = torch::zeros({32, 64, 16}, torch::dtype(torch::kInt64));
  const int rc = vo_fmha_bwd_trace(reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
  TORCH_CHECK(rc == 0, "no traced FMHA backward launch to read (run version 6 first): ", rc);
  return out;
}

}  // namespace vo
