// Compiles the reference's 2:4 microbenchmark (kebab/lib/microbench/
// sparse_mma.cu, included unmodified from the reference tree; its main() is
// renamed away) so that its host-side group-code and ordered-metadata
// encoders can be called from tests. Only host functions are called; the
// file's device kernels are compiled but never launched. Output:
// oracle/_ref/libkebab_ref_sparse_mma.so. Test infrastructure only.
#define main kebab_ref_sparse_mma_main
#include "kebab/lib/microbench/sparse_mma.cu"
#undef main

#include <cstring>

extern "C" {

int kbr_sm_tile_m() { return M; }
int kbr_sm_tile_k() { return K; }

uint32_t kbr_sm_encode_2of4(int i0, int i1) { return encode_2of4(i0, i1); }

void kbr_sm_decode_2of4(uint32_t code, int* i0, int* i1) { decode_2of4(code, *i0, *i1); }

void kbr_sm_prune(const uint16_t* in, uint16_t* out) {
  std::vector<__half> a(M * K), s;
  std::memcpy(a.data(), in, sizeof(uint16_t) * M * K);
  prune_dense_to_sparse_2of4(a, s);
  std::memcpy(out, s.data(), sizeof(uint16_t) * M * K);
}

int kbr_sm_pack(const uint16_t* in, uint16_t* packed, uint32_t* meta) {
  std::vector<__half> a(M * K), p;
  std::vector<uint32_t> m;
  std::memcpy(a.data(), in, sizeof(uint16_t) * M * K);
  if (!encode_sparse_to_packed_and_meta(a, p, m)) return 0;
  std::memcpy(packed, p.data(), sizeof(uint16_t) * M * PACKED_K);
  std::memcpy(meta, m.data(), sizeof(uint32_t) * M * PACKED_K);
  return 1;
}

// codes: M x (K/4) group codes -> M*2 u32 words.
void kbr_sm_meta_rowpair(const uint32_t* codes, uint32_t* out) {
  std::vector<uint32_t> c(codes, codes + M * GROUPS_PER_ROW), o;
  encode_ordered_metadata_rowpair(c, o);
  std::memcpy(out, o.data(), sizeof(uint32_t) * o.size());
}

void kbr_sm_meta_il2(const uint32_t* codes, uint32_t* out) {
  std::vector<uint32_t> c(codes, codes + M * GROUPS_PER_ROW), o;
  encode_ordered_metadata_interleaved2(c, o);
  std::memcpy(out, o.data(), sizeof(uint32_t) * o.size());
}

}  // extern "C"
