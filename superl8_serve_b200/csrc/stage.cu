// s8b_stage_step: one stage step for one micro-batch, enqueued from a plain-pointer
// descriptor (no Python on the path). The launch sequence is the Python stage runtime's
// (StageRunner.run / layer / _moe_ffn), entry point for entry point, so both give identical
// results; see include/s8b.h for the descriptor.
#include "common.cuh"

namespace {

#define S8B_TRY(expr)          \
  do {                         \
    const int rc_ = (expr);    \
    if (rc_ != S8B_OK) return rc_; \
  } while (0)

struct Step {
  const S8bStageDesc &d;
  void *st;
  int M;
  bool tc;  // tensor-core GEMMs (and split-K partials) for this launch size

  // y = dequant(xq @ w^T) in the activation dtype (out_kind 0)
  int gemm(const int8_t *xq, const float *xs, const int8_t *w, const int8_t *packed,
           const float *s, void *y, int N, int K) const {
    if (tc && packed)
      return s8b_gemm_w8a8_tc_packed(xq, xs, packed, s, y, 0, M, N, K, d.dtype, d.tc_ws,
                                     d.tc_ws_bytes, st);
    if (tc)
      return s8b_gemm_w8a8_tc(xq, xs, w, s, y, 0, M, N, K, d.dtype, d.tc_ws, d.tc_ws_bytes, st);
    return s8b_gemm_w8a8(xq, xs, w, s, y, 0, M, N, K, d.dtype, st);
  }
  // split-K partials into d.part; returns the partial count (or a negative status)
  int gemm_split(const int8_t *packed, int N, int K) const {
    const int C = s8b_gemm_tc_split_count(M, N, K);
    if (C < 0) return C;
    const int rc = s8b_gemm_w8a8_tc_packed(d.xq, d.xs, packed, nullptr, d.part, 2, M, N, K,
                                           d.dtype, d.tc_ws, d.tc_ws_bytes, st);
    return rc ? rc : C;
  }
  int rms(const void *h, const void *res_in, const void *w, int C, const float *ws,
          void *y_out) const {
    if (C > 0)
      return s8b_rmsnorm_quant_split(d.part, C, d.xs, ws, res_in, d.res, w, d.eps, d.xq, d.xs,
                                     y_out, M, d.H, d.dtype, st);
    return s8b_rmsnorm_quant(h, res_in, d.res, w, d.eps, d.xq, d.xs, y_out, M, d.H, d.dtype, st);
  }

  int moe(const S8bLayerDesc &L) const {
    const int E = L.moe_experts, k = L.moe_top_k, Fe = L.moe_ffn, A = M * k;
    S8B_TRY(s8b_moe_route(d.moe_y, d.dtype, L.router, M, d.H, E, k, L.moe_norm_topk,
                          L.moe_scaling, d.moe_topi, d.moe_topw, d.moe_offsets,
                          d.moe_sorted_assign, d.moe_sorted_token, d.moe_assign_pos, st));
    S8B_TRY(s8b_moe_gemm_grouped(d.xq, d.xs, d.moe_sorted_token, L.moe_gu_w, L.moe_gu_s,
                                 d.moe_offsets, d.moe_gu, A, 2 * Fe, d.H, E, d.dtype, st));
    S8B_TRY(s8b_silu_mul_quant(d.moe_gu, A, Fe, nullptr, d.moe_aq, d.moe_as, d.dtype, st));
    S8B_TRY(s8b_moe_gemm_grouped(d.moe_aq, d.moe_as, nullptr, L.moe_d_w, L.moe_d_s,
                                 d.moe_offsets, d.moe_contrib, A, d.H, Fe, E, d.dtype, st));
    return s8b_moe_combine(d.moe_contrib, d.moe_topw, d.moe_topi, d.moe_assign_pos, d.h, M, k,
                           d.H, d.dtype, st);
  }

  // One layer. in_C / in_ws: the layer input as split-K partials (C > 0) of the previous down
  // projection, else d.h; codec_in: the layer input is the received boundary payload (the
  // stage prologue). Returns through out_C / out_ws the same for the layer output.
  int layer(int li, bool first_of_model, bool codec_in, int in_C, const float *in_ws,
            bool keep_split, int *out_C, const float **out_ws) const {
    const S8bLayerDesc &L = d.layers[li];
    const int H = d.H, Nqkv = (d.Hq + 2 * d.Hkv) * d.D;
    *out_C = 0;
    *out_ws = nullptr;
    if (codec_in)
      S8B_TRY(s8b_rmsnorm_quant_codec(d.in_payload, d.in_scales, d.scheme, d.res, L.in_norm,
                                      d.eps, d.xq, d.xs, M, H, d.dtype, st));
    else
      S8B_TRY(rms(d.h, first_of_model ? nullptr : d.res, L.in_norm, in_C, in_ws, nullptr));
    if (tc) {
      const int C = gemm_split(L.qkv_packed, Nqkv, H);
      if (C < 0) return C;
      S8B_TRY(s8b_qkv_post_split(d.part, C, d.xs, L.qkv_s, d.positions, d.cos_tab, d.sin_tab,
                                 d.rope_len, L.q_norm, L.k_norm, d.eps, M, d.Hq, d.Hkv, d.D,
                                 d.q_i8, d.q_s, nullptr, L.kc, L.ks, L.vc, L.vs, nullptr,
                                 d.block_table, d.max_blocks, d.block_size, d.dtype, st));
    } else {
      S8B_TRY(gemm(d.xq, d.xs, L.qkv_w, L.qkv_packed, L.qkv_s, d.qkv, Nqkv, H));
      S8B_TRY(s8b_qkv_post(d.qkv, d.positions, d.cos_tab, d.sin_tab, d.rope_len, L.q_norm,
                           L.k_norm, d.eps, M, d.Hq, d.Hkv, d.D, d.q_i8, d.q_s, nullptr, L.kc,
                           L.ks, L.vc, L.vs, nullptr, d.block_table, d.max_blocks,
                           d.block_size, d.dtype, st));
    }
    S8B_TRY(s8b_paged_decode_q8(d.q_i8, d.q_s, L.kc, L.ks, L.vc, L.vs, d.block_table,
                                d.context_lens, d.attn, d.xq, d.xs, M, d.Hq, d.Hkv, d.D,
                                d.block_size, d.max_blocks, d.max_ctx, d.scale, d.attn_ws,
                                d.attn_ws_bytes, d.dtype, st));
    const int Kattn = d.Hq * d.D;
    if (L.moe_experts > 0) {
      if (tc) {
        const int C = gemm_split(L.o_packed, H, Kattn);
        if (C < 0) return C;
        S8B_TRY(rms(nullptr, d.res, L.post_norm, C, L.o_s, d.moe_y));
      } else {
        S8B_TRY(gemm(d.xq, d.xs, L.o_w, L.o_packed, L.o_s, d.h, H, Kattn));
        S8B_TRY(rms(d.h, d.res, L.post_norm, 0, nullptr, d.moe_y));
      }
      return moe(L);
    }
    if (tc) {
      int C = gemm_split(L.o_packed, H, Kattn);
      if (C < 0) return C;
      S8B_TRY(rms(nullptr, d.res, L.post_norm, C, L.o_s, nullptr));
      C = gemm_split(L.gu_packed, 2 * d.F, H);
      if (C < 0) return C;
      S8B_TRY(s8b_silu_mul_quant_split(d.part, C, d.xs, L.gu_s, M, d.F, nullptr, d.xq, d.xs,
                                       d.dtype, st));
      if (keep_split) {
        C = gemm_split(L.d_packed, H, d.F);
        if (C < 0) return C;
        *out_C = C;
        *out_ws = L.d_s;
        return S8B_OK;
      }
      return gemm(d.xq, d.xs, L.d_w, L.d_packed, L.d_s, d.h, H, d.F);
    }
    S8B_TRY(gemm(d.xq, d.xs, L.o_w, L.o_packed, L.o_s, d.h, H, Kattn));
    S8B_TRY(rms(d.h, d.res, L.post_norm, 0, nullptr, nullptr));
    S8B_TRY(gemm(d.xq, d.xs, L.gu_w, L.gu_packed, L.gu_s, d.gu, 2 * d.F, H));
    S8B_TRY(s8b_silu_mul_quant(d.gu, M, d.F, nullptr, d.xq, d.xs, d.dtype, st));
    return gemm(d.xq, d.xs, L.d_w, L.d_packed, L.d_s, d.h, H, d.F);
  }
};

}  // namespace

extern "C" int s8b_stage_step(const S8bStageDesc *desc, void *stream) {
  if (!desc || !desc->layers || !desc->h || !desc->res || !desc->xq || !desc->xs ||
      !desc->q_i8 || !desc->q_s || !desc->attn || !desc->attn_ws || !desc->ids ||
      !desc->positions || !desc->context_lens || !desc->block_table || !desc->cos_tab ||
      !desc->sin_tab)
    return S8B_ERR_ARG;
  const S8bStageDesc &d = *desc;
  if (d.n_layers < 0 || d.M < 0 || d.H <= 0 || d.V <= 0) return S8B_ERR_SHAPE;
  if (d.M == 0) return S8B_OK;
  const bool last = d.head_w != nullptr;
  if (!d.embed && (!d.in_payload || !d.in_scales)) return S8B_ERR_ARG;
  if (!last && (!d.out_payload || !d.out_scales)) return S8B_ERR_ARG;
  const bool tc = d.tc_min > 0 && d.M >= d.tc_min && d.part && d.tc_ws;
  for (int li = 0; li < d.n_layers; ++li) {
    const S8bLayerDesc &L = d.layers[li];
    if (tc && (!L.qkv_packed || !L.o_packed)) return S8B_ERR_ARG;
    if (!tc && !d.qkv) return S8B_ERR_ARG;
    if (L.moe_experts > 0) {
      if (!L.router || !L.moe_gu_w || !L.moe_d_w || !d.moe_y || !d.moe_topi ||
          !d.moe_contrib || !d.moe_aq)
        return S8B_ERR_ARG;
    } else {
      if (!L.gu_w || !L.d_w || (!tc && !d.gu) || (tc && (!L.gu_packed || !L.d_packed)))
        return S8B_ERR_ARG;
    }
  }
  Step s{d, stream, d.M, tc};
  // stage prologue: the first RMSNorm decodes the received [hidden | residual] on load
  if (d.embed)
    S8B_TRY(s8b_embed(d.ids, d.embed, d.M, d.H, d.h, d.dtype, stream));
  else if (d.n_layers == 0)
    S8B_TRY(s8b_codec_decode(d.in_payload, d.in_scales, d.M, d.H, d.H, d.scheme, d.h, d.res,
                             d.dtype, stream));
  int C = 0;
  const float *ws = nullptr;
  for (int li = 0; li < d.n_layers; ++li) {
    int oc = 0;
    const float *ow = nullptr;
    S8B_TRY(s.layer(li, d.first_model_layer && li == 0, li == 0 && !d.embed, C, ws, true, &oc,
                    &ow));
    C = oc;
    ws = ow;
  }
  // stage epilogue: the encoder reduces the last down projection's split-K partials
  if (!last && C > 0)
    return s8b_codec_encode_split(d.part, C, d.xs, ws, d.res, d.M, d.H, d.H, d.scheme,
                                  d.out_payload, d.out_scales, d.dtype, stream);
  if (!last)
    return s8b_codec_encode(d.h, d.res, d.M, d.H, d.H, d.scheme, d.out_payload, d.out_scales,
                            d.dtype, stream);
  if (!d.head) return S8B_OK;
  if (!d.final_norm || !d.logits) return S8B_ERR_ARG;
  S8B_TRY(s.rms(d.h, d.res, d.final_norm, C, ws, nullptr));
  S8B_TRY(s.gemm(d.xq, d.xs, d.head_w, d.head_packed, d.head_s, d.logits, d.V, d.H));
  if (!d.temperature) return s8b_argmax(d.logits, d.M, d.V, d.ids, d.dtype, stream);
  return s8b_sample(d.logits, d.dtype, d.M, d.V, d.temperature, d.top_k, d.top_p, d.penalty,
                    d.input_ids, d.positions, d.history, d.history_cap, d.seeds, d.sample_ws,
                    d.sample_ws_bytes, d.ids, stream);
}

extern "C" size_t s8b_stage_desc_size(void) { return sizeof(S8bStageDesc); }
extern "C" size_t s8b_layer_desc_size(void) { return sizeof(S8bLayerDesc); }
