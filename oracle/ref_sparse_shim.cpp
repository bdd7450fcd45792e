// Compiles the reference's host-side 2:4 prune / pack / CUTLASS-metadata
// functions (kebab/lib/microbench/cutlass_meta_probe.cu, included unmodified
// from the reference tree; its main() is renamed away) into
// oracle/_ref/libkebab_ref_sparse.so. They work on the probe's fixed 16 x 32
// tile. Test infrastructure only: used to pin kebab_oracle.cpp's packers.
#define main kebab_ref_cutlass_meta_probe_main
#include "kebab/lib/microbench/cutlass_meta_probe.cu"
#undef main

#include <cstring>

extern "C" {

int kbr_tile_m() { return M; }
int kbr_tile_k() { return K; }

// prune_dense_to_sparse_2of4 on one 16 x 32 FP16 tile (row-major).
void kbr_prune_16x32(const uint16_t* in, uint16_t* out) {
  std::vector<__half> a(M * K), s;
  std::memcpy(a.data(), in, sizeof(uint16_t) * M * K);
  prune_dense_to_sparse_2of4(a, s);
  std::memcpy(out, s.data(), sizeof(uint16_t) * M * K);
}

// encode_sparse_to_packed_and_meta: returns 1 on success, 0 on failure.
int kbr_pack_16x32(const uint16_t* in, uint16_t* packed, uint32_t* meta) {
  std::vector<__half> a(M * K), p;
  std::vector<uint32_t> m;
  std::memcpy(a.data(), in, sizeof(uint16_t) * M * K);
  bool ok = encode_sparse_to_packed_and_meta(a, p, m);
  if (!ok) return 0;
  std::memcpy(packed, p.data(), sizeof(uint16_t) * M * PACKED_K);
  std::memcpy(meta, m.data(), sizeof(uint32_t) * M * PACKED_K);
  return 1;
}

// encode_cutlass_metadata_interleaved2: 16 x 16 positions -> 64 u32 slots.
void kbr_meta_cutlass_16x32(const uint32_t* meta, uint32_t* out) {
  std::vector<uint32_t> m(meta, meta + M * PACKED_K), o;
  encode_cutlass_metadata_interleaved2(m, o);
  std::memcpy(out, o.data(), sizeof(uint32_t) * o.size());
}

void kbr_meta_cutlass_decode_16x32(const uint32_t* enc, uint32_t* meta) {
  std::vector<uint32_t> e(enc, enc + M * 4), o;
  decode_cutlass_metadata_interleaved2(e, o);
  std::memcpy(meta, o.data(), sizeof(uint32_t) * o.size());
}

uint32_t kbr_encode_2of4(int i0, int i1) { return encode_2of4(i0, i1); }

// The reference probe's own main (its self-check), returning its exit code.
int kbr_probe_main() { return kebab_ref_cutlass_meta_probe_main(); }

}  // extern "C"
