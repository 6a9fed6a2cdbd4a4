// container.cpp -- BOA2 chunked container: serialise and parse.
//
// Same on-disk layout as the reference writer and reader (compress_v2,
// boa.cpp:538-581; read_boa2, boa.cpp:190-277), so files are interchangeable:
//   "BOA2" | u32 version=1 | u32 flags | u64 total | u32 chunk_len |
//   u32 n_chunks | u32 last_chunk_len | u8 fp_len | fp | payload |
//   "IDX2" first_bytes[n] uvarint(len)[n] | u32 CRC-32(IDX2..)
// The parser also accepts the older IDX1 index (delta offsets + lengths) and
// reports malformed input as BOA_E_FORMAT instead of aborting.
#include <cstring>
#include <vector>

#include "../../include/boa_b200.h"

namespace {

uint32_t crc32_table_entry(uint32_t i) {
  uint32_t c = i;
  for (int k = 0; k < 8; ++k) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
  return c;
}
struct Crc32 {
  uint32_t t[256];
  Crc32() { for (uint32_t i = 0; i < 256; ++i) t[i] = crc32_table_entry(i); }
  uint32_t operator()(const uint8_t* p, size_t n) const {
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) c = t[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
  }
};
const Crc32& crc32() {
  static const Crc32 c;
  return c;
}

void put_uvarint(std::vector<uint8_t>& o, uint64_t x) {
  do {
    uint8_t b = (uint8_t)(x & 0x7Fu);
    x >>= 7;
    o.push_back((uint8_t)(b | (x ? 0x80u : 0u)));
  } while (x);
}
bool get_uvarint(const uint8_t* buf, size_t end, size_t& pos, uint64_t& x) {
  x = 0;
  for (int shift = 0; shift < 64; shift += 7) {
    if (pos >= end) return false;
    const uint8_t b = buf[pos++];
    x |= (uint64_t)(b & 0x7Fu) << shift;
    if (!(b & 0x80u)) return true;
  }
  return false;
}
template <class T>
void put(std::vector<uint8_t>& o, T v) {
  uint8_t b[sizeof(T)];
  std::memcpy(b, &v, sizeof(T));
  o.insert(o.end(), b, b + sizeof(T));
}
template <class T>
T get(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

}  // namespace

extern "C" {

int boa_boa2_build(uint64_t total, uint32_t chunk_len, uint32_t n_chunks, uint32_t last_len, uint32_t flags,
                   uint32_t interleave, const uint8_t* first_bytes, const uint64_t* stream_bytes,
                   const uint8_t* payload, uint8_t* buf, size_t cap, size_t* len_out) {
  uint8_t fp[4];
  std::memcpy(fp, &interleave, 4);
  return boa_boa2_build_fp(total, chunk_len, n_chunks, last_len, flags, fp, (flags & 1u) ? 4 : 0, first_bytes,
                           stream_bytes, payload, buf, cap, len_out);
}

int boa_boa2_build_fp(uint64_t total, uint32_t chunk_len, uint32_t n_chunks, uint32_t last_len, uint32_t flags,
                      const uint8_t* fp, uint32_t fp_len, const uint8_t* first_bytes, const uint64_t* stream_bytes,
                      const uint8_t* payload, uint8_t* buf, size_t cap, size_t* len_out) {
  if (!len_out || (n_chunks && (!first_bytes || !stream_bytes))) return BOA_E_INVALID;
  if (fp_len > 255 || (fp_len && !fp)) return BOA_E_INVALID;
  uint64_t pay = 0;
  for (uint32_t i = 0; i < n_chunks; ++i) pay += stream_bytes[i];
  if (pay && !payload) return BOA_E_INVALID;
  std::vector<uint8_t> head, idx;
  head.insert(head.end(), {'B', 'O', 'A', '2'});
  put<uint32_t>(head, 1u);
  put<uint32_t>(head, flags);
  put<uint64_t>(head, total);
  put<uint32_t>(head, chunk_len);
  put<uint32_t>(head, n_chunks);
  put<uint32_t>(head, last_len);
  head.push_back((uint8_t)fp_len);
  head.insert(head.end(), fp, fp + fp_len);
  idx.insert(idx.end(), {'I', 'D', 'X', '2'});
  idx.insert(idx.end(), first_bytes, first_bytes + n_chunks);
  for (uint32_t i = 0; i < n_chunks; ++i) put_uvarint(idx, stream_bytes[i]);
  const uint32_t crc = crc32()(idx.data(), idx.size());
  const size_t need = head.size() + pay + idx.size() + 4;
  *len_out = need;
  if (!buf) return BOA_OK;
  if (cap < need) return BOA_E_INVALID;
  uint8_t* p = buf;
  std::memcpy(p, head.data(), head.size()); p += head.size();
  if (pay) { std::memcpy(p, payload, pay); p += pay; }
  std::memcpy(p, idx.data(), idx.size()); p += idx.size();
  std::memcpy(p, &crc, 4);
  return BOA_OK;
}

int boa_boa2_parse(const uint8_t* buf, size_t len, boa2_info* info, uint8_t* first_bytes, uint64_t* offsets,
                   uint64_t* lengths) {
  if (!buf || !info) return BOA_E_INVALID;
  if (len < 33) return BOA_E_FORMAT;
  if (std::memcmp(buf, "BOA2", 4) != 0) return BOA_E_FORMAT;
  if (get<uint32_t>(buf + 4) != 1u) return BOA_E_FORMAT;
  boa2_info I{};
  I.flags = get<uint32_t>(buf + 8);
  I.total_size = get<uint64_t>(buf + 12);
  I.chunk_len = get<uint32_t>(buf + 20);
  I.n_chunks = get<uint32_t>(buf + 24);
  I.last_chunk_len = get<uint32_t>(buf + 28);
  size_t p = 32;
  const uint8_t fp_len = buf[p++];
  if (p + fp_len > len) return BOA_E_FORMAT;
  if ((I.flags & 1u) && fp_len >= 4) I.interleave_batch = get<uint32_t>(buf + p);
  I.fp_len = fp_len;
  std::memcpy(I.fp, buf + p, fp_len);
  p += fp_len;
  I.payload_offset = p;
  // backward scan for the index marker (boa.cpp:218-225)
  size_t idx = (size_t)-1;
  for (size_t i = len - 4; i-- > p;) {
    if (buf[i] == 'I' && buf[i + 1] == 'D' && buf[i + 2] == 'X' && (buf[i + 3] == '2' || buf[i + 3] == '1')) {
      idx = i;
      I.index_version = buf[i + 3] - '0';
      break;
    }
  }
  if (idx == (size_t)-1 || len < idx + 8) return BOA_E_FORMAT;
  if (get<uint32_t>(buf + len - 4) != crc32()(buf + idx, len - idx - 4)) return BOA_E_FORMAT;
  I.payload_bytes = idx - p;
  const size_t end = len - 4;
  size_t q = idx + 4;
  if (q + I.n_chunks > end) return BOA_E_FORMAT;
  if (first_bytes) std::memcpy(first_bytes, buf + q, I.n_chunks);
  q += I.n_chunks;
  std::vector<uint64_t> off(I.n_chunks), ln(I.n_chunks);
  if (I.index_version == 1) {
    uint64_t prev = 0, dlt;
    for (uint32_t i = 0; i < I.n_chunks; ++i) {
      if (!get_uvarint(buf, end, q, dlt)) return BOA_E_FORMAT;
      prev += dlt;
      off[i] = prev;
    }
    for (uint32_t i = 0; i < I.n_chunks; ++i)
      if (!get_uvarint(buf, end, q, ln[i])) return BOA_E_FORMAT;
  } else {
    uint64_t o = 0;
    for (uint32_t i = 0; i < I.n_chunks; ++i) {
      if (!get_uvarint(buf, end, q, ln[i])) return BOA_E_FORMAT;
      off[i] = o;
      o += ln[i];
    }
  }
  for (uint32_t i = 0; i < I.n_chunks; ++i)
    if (off[i] + ln[i] > I.payload_bytes) return BOA_E_FORMAT;  // boa.cpp:268
  if (offsets) std::memcpy(offsets, off.data(), off.size() * 8);
  if (lengths) std::memcpy(lengths, ln.data(), ln.size() * 8);
  *info = I;
  return BOA_OK;
}

}  // extern "C"
