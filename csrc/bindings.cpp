// Python bindings of the vllm_moet_b200 native library (_C).
#include <torch/extension.h>

// runtime/pack_io.cpp
void register_pack_io(pybind11::module& m);
// norm_quant.cu
void rmsnorm_quant(torch::Tensor x, c10::optional<torch::Tensor> add, c10::optional<torch::Tensor> x_out,
                   torch::Tensor w, double eps, c10::optional<torch::Tensor> y_out,
                   c10::optional<torch::Tensor> q0, c10::optional<torch::Tensor> s0,
                   c10::optional<torch::Tensor> q1, c10::optional<torch::Tensor> s1, int64_t ostride,
                   c10::optional<torch::Tensor> ar);
void swiglu_quant(torch::Tensor in, double limit, c10::optional<torch::Tensor> n_rows, int64_t layout,
                  torch::Tensor q, torch::Tensor s);
void quant_fp8(torch::Tensor x, int64_t layout, torch::Tensor q, torch::Tensor s);
// gemv_fp8.cu
void gemv_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
              c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> ar);
// moe_route.cu
void router_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t k, bool sigmoid,
                 int64_t n_group, int64_t topk_group, bool norm, double scaling, torch::Tensor ids,
                 torch::Tensor wts);
void build_pairs(torch::Tensor topk_ids, int64_t E, int64_t MB, torch::Tensor rank_scratch,
                 torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                 torch::Tensor status, int64_t e_lo);
void router_logits(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> part,
                   c10::optional<torch::Tensor> cnt);
void moe_route_fused(torch::Tensor x, torch::Tensor w, torch::Tensor logits, c10::optional<torch::Tensor> bias,
                     int64_t k, bool sigmoid, int64_t n_group, int64_t topk_group, bool norm, double scaling,
                     torch::Tensor ids, torch::Tensor wts, int64_t MB, torch::Tensor rank_scratch,
                     torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                     torch::Tensor counter, torch::Tensor status, int64_t e_lo, int64_t E_local);
void mla_combine_uv(torch::Tensor o_part, torch::Tensor ml_part, torch::Tensor wuv, torch::Tensor swuv,
                    torch::Tensor q, torch::Tensor qs);
void argmax_split(torch::Tensor logits, c10::optional<torch::Tensor> ids, c10::optional<torch::Tensor> lse,
                  c10::optional<torch::Tensor> status, torch::Tensor part, torch::Tensor counter,
                  c10::optional<torch::Tensor> mv, int64_t id_offset);
void argmax_merge(torch::Tensor parts, torch::Tensor ids);
void argmax_merge_ar(torch::Tensor mv, torch::Tensor ids, torch::Tensor ar);
void build_pairs_padded(torch::Tensor topk_ids, int64_t E, int64_t MB, torch::Tensor rank_scratch,
                        torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                        torch::Tensor n_rows, torch::Tensor status, int64_t e_lo);
void gather_rows(torch::Tensor src_q, torch::Tensor src_s, torch::Tensor idx, torch::Tensor n_rows, torch::Tensor dst_q,
                 torch::Tensor dst_s);
// moe_w2.cu
void moe_w2_gemv(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
                 torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
                 torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t rows_per_pair,
                 c10::optional<torch::Tensor> miss_count, c10::optional<torch::Tensor> pool8, int64_t codes_off8,
                 int64_t scale_off8, c10::optional<torch::Tensor> slot_table8, bool quintal,
                 c10::optional<torch::Tensor> ep, c10::optional<torch::Tensor> ret_rows);
void ep_dispatch(torch::Tensor desc, torch::Tensor xq, torch::Tensor xs, torch::Tensor ids);
void ep_recv_pairs(torch::Tensor desc, int64_t MB, torch::Tensor ids, torch::Tensor rank_scratch,
                   torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                   torch::Tensor n_rows);
int64_t ep_buffer_bytes(int64_t world, int64_t cap, int64_t H);
void experts_quant_pack(torch::Tensor w, torch::Tensor ts, torch::Tensor packed, torch::Tensor sf,
                        torch::Tensor counters, torch::Tensor pool, int64_t off_c, int64_t off_s, int64_t zero_mode);
void moe_w2_tcd(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
                torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
                torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t rows_per_pair,
                c10::optional<torch::Tensor> miss_count, torch::Tensor status);
void moe_combine(torch::Tensor y, torch::Tensor pos_of, torch::Tensor wts, c10::optional<torch::Tensor> resid,
                 c10::optional<torch::Tensor> shared_out, c10::optional<torch::Tensor> out,
                 c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> ar,
                 c10::optional<torch::Tensor> ep);
// gemv_stream.cu
void gemv_stream_fp8(c10::optional<torch::Tensor> a, c10::optional<torch::Tensor> sa, torch::Tensor w,
                     torch::Tensor sw, torch::Tensor out, c10::optional<torch::Tensor> resid, torch::Tensor status,
                     c10::optional<torch::Tensor> x_norm, c10::optional<torch::Tensor> gamma, double eps,
                     c10::optional<torch::Tensor> x_add, c10::optional<torch::Tensor> x_out,
                     c10::optional<torch::Tensor> ar_push, c10::optional<torch::Tensor> ar_consume);
// indexer.cu
void indexer_logits(torch::Tensor q, torch::Tensor w, torch::Tensor k_cache, torch::Tensor block_table,
                    torch::Tensor seq_of_tok, torch::Tensor pos_of_tok, torch::Tensor out, torch::Tensor status);
void indexer_topk(torch::Tensor scores, int64_t k, torch::Tensor out);
void idx_k_write(torch::Tensor k, torch::Tensor slot, torch::Tensor cache, torch::Tensor status);
// bf12.cu
void bf12_decode(torch::Tensor cls, torch::Tensor lo, torch::Tensor lut, torch::Tensor esc_pos, torch::Tensor esc_hi,
                 torch::Tensor out);
// symm.cu
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t bytes);
int64_t symm_open(at::Tensor handle);
void symm_close(int64_t ptr);
void symm_free(int64_t ptr);
at::Tensor symm_view(int64_t ptr, int64_t bytes, int64_t device);
void ar_test(at::Tensor desc, at::Tensor x, c10::optional<at::Tensor> resid, at::Tensor out, int64_t mode);

// mla_decode.cu
void mla_decode(torch::Tensor q, torch::Tensor kv, torch::Tensor block_table, torch::Tensor seq_of_tok,
                torch::Tensor pos_of_tok, torch::Tensor o_part, torch::Tensor ml_part, double scale,
                torch::Tensor status, c10::optional<torch::Tensor> sel);
void mla_combine(torch::Tensor o_part, torch::Tensor ml_part, c10::optional<torch::Tensor> out,
                 c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs);
// mla_prep.cu
void q_prep(torch::Tensor qb, int64_t Hh, int64_t nope, int64_t rope, torch::Tensor pos_of_tok,
            torch::Tensor cos_sin, c10::optional<torch::Tensor> qn_q, c10::optional<torch::Tensor> qn_s,
            c10::optional<torch::Tensor> qcat, int64_t rope_off, c10::optional<torch::Tensor> q_out);
void kv_prep(torch::Tensor kva, int64_t lat, int64_t rope, torch::Tensor norm_w, double eps, torch::Tensor pos_of_tok,
             torch::Tensor cos_sin, c10::optional<torch::Tensor> slot_mapping, int64_t cache_mode,
             c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> lat_out,
             c10::optional<torch::Tensor> rope_out, c10::optional<torch::Tensor> lat_q,
             c10::optional<torch::Tensor> lat_s, torch::Tensor status);
// mla_prefill.cu
void mla_prefill(torch::Tensor q, torch::Tensor kvb, torch::Tensor kr, torch::Tensor cu_seqlens, int64_t max_len,
                 double scale, c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_s,
                 c10::optional<torch::Tensor> out_bf16, c10::optional<torch::Tensor> cu_seqlens_k);
// trellis.cu
void trellis_rot_in(torch::Tensor x, torch::Tensor src, torch::Tensor eid, torch::Tensor su, torch::Tensor out);
void trellis_rot_out(torch::Tensor z, torch::Tensor eid, torch::Tensor sv, c10::optional<torch::Tensor> scale,
                     torch::Tensor out);
void trellis_gemv(torch::Tensor xr, torch::Tensor trellis, torch::Tensor experts, torch::Tensor row_map,
                  torch::Tensor z, int64_t K, int64_t L, bool mad, double inv_rms, int64_t maxr);
// hyper_conn.cu
void hc_mix(torch::Tensor xs, c10::optional<torch::Tensor> upd, c10::optional<torch::Tensor> post,
            c10::optional<torch::Tensor> comb, c10::optional<torch::Tensor> fn, c10::optional<torch::Tensor> part);
void hc_apply(torch::Tensor xs, torch::Tensor part, torch::Tensor base, torch::Tensor scale, double eps,
              int64_t iters, double rms_eps, torch::Tensor h, c10::optional<torch::Tensor> post,
              c10::optional<torch::Tensor> comb);
// quant_pack.cu
void nvfp4_quant(torch::Tensor w, double ts, torch::Tensor packed, torch::Tensor sf);
void w2_quant_pack(torch::Tensor packed, torch::Tensor sf, double ts, int64_t zero_mode, torch::Tensor codes_plane,
                   torch::Tensor scale_plane, c10::optional<torch::Tensor> fp4_plane,
                   c10::optional<torch::Tensor> counters);
// sampling.cu
void argmax_lse(torch::Tensor logits, torch::Tensor ids, c10::optional<torch::Tensor> lse,
                c10::optional<torch::Tensor> maxv, c10::optional<torch::Tensor> status);
void mtp_accept(torch::Tensor targets, torch::Tensor tokens, torch::Tensor out_tokens, torch::Tensor n_acc,
                c10::optional<torch::Tensor> active);
void mtp_finalize(torch::Tensor targets, torch::Tensor n_acc, torch::Tensor drafts, torch::Tensor tokens,
                  torch::Tensor seq_pos, c10::optional<torch::Tensor> active);

void tc_moe_w2(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
               torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
               torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t nt,
               c10::optional<torch::Tensor> miss_count, torch::Tensor status, int64_t dbg);
void tc_gemm_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
                 c10::optional<torch::Tensor> resid, int64_t nt, torch::Tensor status);

void ws_moe_w2(torch::Tensor a, torch::Tensor sa, torch::Tensor pairs, torch::Tensor n_pairs, torch::Tensor pool,
               int64_t codes_off, int64_t scale_off, torch::Tensor slot_table, torch::Tensor out, int64_t N,
               int64_t K, int64_t nt, c10::optional<torch::Tensor> miss_count, torch::Tensor status,
               c10::optional<torch::Tensor> dbg_clk);
void ws_gemm_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
                 c10::optional<torch::Tensor> resid, int64_t T, torch::Tensor status);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_pack_io(m);
#ifdef MOET_SOURCE_FINGERPRINT
  m.attr("source_fingerprint") = MOET_SOURCE_FINGERPRINT;
#endif
  m.doc() = "vllm_moet_b200 sm_100a kernels";
  m.def("rmsnorm_quant", &rmsnorm_quant, py::arg("x"), py::arg("add"), py::arg("x_out"), py::arg("w"), py::arg("eps"),
        py::arg("y_out"), py::arg("q0"), py::arg("s0"), py::arg("q1"), py::arg("s1"), py::arg("ostride"),
        py::arg("ar") = py::none());
  m.def("swiglu_quant", &swiglu_quant);
  m.def("quant_fp8", &quant_fp8);
  m.def("gemv_fp8", &gemv_fp8, py::arg("a"), py::arg("sa"), py::arg("w"), py::arg("sw"), py::arg("out"),
        py::arg("resid"), py::arg("ar") = py::none());
  m.def("router_topk", &router_topk);
  m.def("build_pairs", &build_pairs, py::arg("topk_ids"), py::arg("E"), py::arg("MB"), py::arg("rank_scratch"),
        py::arg("sorted_tok"), py::arg("pos_of"), py::arg("pairs"), py::arg("n_pairs"), py::arg("status"),
        py::arg("e_lo") = -1);
  m.def("build_pairs_padded", &build_pairs_padded, py::arg("topk_ids"), py::arg("E"), py::arg("MB"),
        py::arg("rank_scratch"), py::arg("sorted_tok"), py::arg("pos_of"), py::arg("pairs"), py::arg("n_pairs"),
        py::arg("n_rows"), py::arg("status"), py::arg("e_lo") = -1);
  m.def("gather_rows", &gather_rows);
  m.def("router_logits", &router_logits, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("part") = py::none(),
        py::arg("cnt") = py::none());
  m.def("moe_route_fused", &moe_route_fused, py::arg("x"), py::arg("w"), py::arg("logits"), py::arg("bias"),
        py::arg("k"), py::arg("sigmoid"), py::arg("n_group"), py::arg("topk_group"), py::arg("norm"),
        py::arg("scaling"), py::arg("ids"), py::arg("wts"), py::arg("MB"), py::arg("rank_scratch"),
        py::arg("sorted_tok"), py::arg("pos_of"), py::arg("pairs"), py::arg("n_pairs"), py::arg("counter"),
        py::arg("status"), py::arg("e_lo") = 0, py::arg("E_local") = 0);
  m.def("mla_combine_uv", &mla_combine_uv);
  m.def("tc_moe_w2", &tc_moe_w2);
  m.def("tc_gemm_fp8", &tc_gemm_fp8);
  m.def("ws_moe_w2", &ws_moe_w2);
  m.def("ws_gemm_fp8", &ws_gemm_fp8);
  m.def("argmax_split", &argmax_split, py::arg("logits"), py::arg("ids"), py::arg("lse"), py::arg("status"),
        py::arg("part"), py::arg("counter"), py::arg("mv") = py::none(), py::arg("id_offset") = 0);
  m.def("argmax_merge", &argmax_merge);
  m.def("argmax_merge_ar", &argmax_merge_ar);
  m.def("moe_w2_gemv", &moe_w2_gemv, py::arg("a"), py::arg("sa"), py::arg("gather"), py::arg("pairs"),
        py::arg("n_pairs"), py::arg("pool"), py::arg("codes_off"), py::arg("scale_off"), py::arg("slot_table"),
        py::arg("out"), py::arg("N"), py::arg("K"), py::arg("rows_per_pair"), py::arg("miss_count"),
        py::arg("pool8") = py::none(), py::arg("codes_off8") = 0, py::arg("scale_off8") = 0,
        py::arg("slot_table8") = py::none(), py::arg("quintal") = false, py::arg("ep") = py::none(),
        py::arg("ret_rows") = py::none());
  m.def("moe_w2_tcd", &moe_w2_tcd);
  m.def("experts_quant_pack", &experts_quant_pack);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_recv_pairs", &ep_recv_pairs);
  m.def("ep_buffer_bytes", &ep_buffer_bytes);
  m.def("moe_combine", &moe_combine, py::arg("y"), py::arg("pos_of"), py::arg("wts"), py::arg("resid"),
        py::arg("shared_out"), py::arg("out"), py::arg("out_f32"), py::arg("ar") = py::none(),
        py::arg("ep") = py::none());
  m.def("bf12_decode", &bf12_decode);
  m.def("indexer_logits", &indexer_logits);
  m.def("indexer_topk", &indexer_topk);
  m.def("gemv_stream_fp8", &gemv_stream_fp8, py::arg("a"), py::arg("sa"), py::arg("w"), py::arg("sw"), py::arg("out"),
        py::arg("resid"), py::arg("status"), py::arg("x_norm") = py::none(), py::arg("gamma") = py::none(),
        py::arg("eps") = 1e-6, py::arg("x_add") = py::none(), py::arg("x_out") = py::none(),
        py::arg("ar_push") = py::none(), py::arg("ar_consume") = py::none());
  m.def("idx_k_write", &idx_k_write);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("symm_view", &symm_view);
  m.def("ar_test", &ar_test);
  m.def("mla_decode", &mla_decode, py::arg("q"), py::arg("kv"), py::arg("block_table"), py::arg("seq_of_tok"),
        py::arg("pos_of_tok"), py::arg("o_part"), py::arg("ml_part"), py::arg("scale"), py::arg("status"),
        py::arg("sel") = py::none());
  m.def("mla_combine", &mla_combine);
  m.def("q_prep", &q_prep);
  m.def("kv_prep", &kv_prep);
  m.def("trellis_rot_in", &trellis_rot_in);
  m.def("trellis_rot_out", &trellis_rot_out, py::arg("z"), py::arg("eid"), py::arg("sv"), py::arg("scale"),
        py::arg("out"));
  m.def("trellis_gemv", &trellis_gemv);
  m.def("hc_mix", &hc_mix, py::arg("xs"), py::arg("upd") = py::none(), py::arg("post") = py::none(),
        py::arg("comb") = py::none(), py::arg("fn") = py::none(), py::arg("part") = py::none());
  m.def("hc_apply", &hc_apply, py::arg("xs"), py::arg("part"), py::arg("base"), py::arg("scale"), py::arg("eps"),
        py::arg("iters"), py::arg("rms_eps"), py::arg("h"), py::arg("post") = py::none(), py::arg("comb") = py::none());
  m.def("mla_prefill", &mla_prefill, py::arg("q"), py::arg("kvb"), py::arg("kr"), py::arg("cu_seqlens"),
        py::arg("max_len"), py::arg("scale"), py::arg("out_q"), py::arg("out_s"), py::arg("out_bf16"),
        py::arg("cu_seqlens_k") = py::none());
  m.def("nvfp4_quant", &nvfp4_quant);
  m.def("w2_quant_pack", &w2_quant_pack);
  m.def("argmax_lse", &argmax_lse);
  m.def("mtp_accept", &mtp_accept);
  m.def("mtp_finalize", &mtp_finalize);
}
