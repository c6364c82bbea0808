// Binary control-protocol frames (see hcp_host.h for the layout).
//
// The message set is the reference's WorkerCommand / WorkerResponse (rust/src/distributed/
// protocol.rs:14-192) minus the NIXL metadata exchange; the reference encodes them with bincode
// over QUIC, here they are fixed little-endian layouts carried by the torch.distributed control
// group. The type ids and field lists below are this framework's own wire format.
#include "hcp_host.h"

#include <cstring>

namespace hcp::host {

namespace {

struct Schema {
  int type;
  const char* kinds;
};

// commands 1-8, responses 64-69
constexpr Schema kSchemas[] = {
    {1, "iAAsiObb"},   // Prefill: request_id, prompt, chunks, strategy, decode_horizon,
                       //          capacity_tickets?, keep_kv, want_logits
    {2, "ii"},         // Decode: request_id, token
    {3, "Pb"},         // DecodeBatch: (request_id, token) rows, want_logits
    {4, "iAAAiib"},    // StationaryContinuation: request_id, tokens, position_ids, tickets, starter,
                       //                         decode_horizon, want_logits
    {5, "iiiAiii"},    // StationaryDecode: request_id, token, position, tickets, starter,
                       //                   token_offset, decode_horizon
    {6, "ii"},         // SyncGlobalSeqLen: request_id, len
    {7, "i"},          // ReleaseRequest: request_id
    {8, ""},           // Shutdown
    {64, "iiiG"},      // PrefillDone: request_id, token, global_seq_len, logits?
    {65, "ii"},        // DecodeDone: request_id, token
    {66, "P"},         // DecodeBatchDone: (request_id, token) rows
    {67, "io"},        // StationaryContinuationDone: request_id, token?
    {68, "i"},         // Ack: request_id
    {69, "is"},        // Error: request_id, message
};

constexpr uint64_t kMaxArray = uint64_t(1) << 32;  // sanity bound on decoded counts

class Writer {
 public:
  template <class T>
  void Put(const T& v) {
    const size_t o = buf.size();
    buf.resize(o + sizeof(T));
    std::memcpy(&buf[o], &v, sizeof(T));
  }
  void Bytes(const void* p, size_t n) {
    const size_t o = buf.size();
    buf.resize(o + n);
    if (n) std::memcpy(&buf[o], p, n);
  }
  std::string buf;
};

class Reader {
 public:
  Reader(const char* p, size_t n) : p_(p), n_(n) {}
  template <class T>
  T Get() {
    Need(sizeof(T));
    T v;
    std::memcpy(&v, p_ + o_, sizeof(T));
    o_ += sizeof(T);
    return v;
  }
  void Bytes(void* dst, size_t n) {
    Need(n);
    if (n) std::memcpy(dst, p_ + o_, n);
    o_ += n;
  }
  uint64_t Count(size_t elem) {
    const uint64_t c = Get<uint64_t>();
    if (c > kMaxArray || c * elem > n_ - o_) throw ProtocolError("array count past the frame end");
    return c;
  }
  bool Done() const { return o_ == n_; }

 private:
  void Need(size_t n) {
    if (n > n_ - o_) throw ProtocolError("field past the frame end");
  }
  const char* p_;
  size_t n_, o_ = 0;
};

}  // namespace

const char* MessageSchema(int type) {
  for (const auto& s : kSchemas)
    if (s.type == type) return s.kinds;
  return "";
}

static bool KnownType(int type) {
  for (const auto& s : kSchemas)
    if (s.type == type) return true;
  return false;
}

std::string EncodeFrame(int type, const std::vector<Field>& fields) {
  if (!KnownType(type)) throw ProtocolError("not a protocol message type: " + std::to_string(type));
  const std::string kinds = MessageSchema(type);
  if (kinds.size() != fields.size())
    throw ProtocolError("message type " + std::to_string(type) + " takes " +
                        std::to_string(kinds.size()) + " fields, got " +
                        std::to_string(fields.size()));
  Writer w;
  w.Put<uint32_t>(0);  // payload size, patched below
  w.Put<uint8_t>(kProtocolVersion);
  w.Put<uint8_t>(uint8_t(type));
  for (size_t k = 0; k < kinds.size(); ++k) {
    const Field& f = fields[k];
    switch (FieldKind(kinds[k])) {
      case FieldKind::kI64: w.Put<int64_t>(f.i); break;
      case FieldKind::kF64: w.Put<double>(f.f); break;
      case FieldKind::kBool: w.Put<uint8_t>(f.i ? 1 : 0); break;
      case FieldKind::kStr:
        if (f.s.size() > 0xffffffffull) throw ProtocolError("string too long");
        w.Put<uint32_t>(uint32_t(f.s.size()));
        w.Bytes(f.s.data(), f.s.size());
        break;
      case FieldKind::kPairs:
        if (f.a.size() % 2) throw ProtocolError("pairs field needs an even number of values");
        w.Put<uint64_t>(f.a.size() / 2);
        w.Bytes(f.a.data(), f.a.size() * sizeof(int64_t));
        break;
      case FieldKind::kOptI64:
        w.Put<uint8_t>(f.present ? 1 : 0);
        if (f.present) w.Put<int64_t>(f.i);
        break;
      case FieldKind::kOptI64Array:
        w.Put<uint8_t>(f.present ? 1 : 0);
        if (!f.present) break;
        [[fallthrough]];
      case FieldKind::kI64Array:
        w.Put<uint64_t>(f.a.size());
        w.Bytes(f.a.data(), f.a.size() * sizeof(int64_t));
        break;
      case FieldKind::kOptF32Array:
        w.Put<uint8_t>(f.present ? 1 : 0);
        if (f.present) {
          w.Put<uint64_t>(f.fa.size());
          w.Bytes(f.fa.data(), f.fa.size() * sizeof(float));
        }
        break;
    }
  }
  const uint64_t payload = w.buf.size() - sizeof(uint32_t);
  if (payload > 0xffffffffull) throw ProtocolError("frame larger than 4 GiB");
  const uint32_t p32 = uint32_t(payload);
  std::memcpy(&w.buf[0], &p32, sizeof(p32));
  return std::move(w.buf);
}

std::vector<Field> DecodeFrame(const std::string& frame, int* type) {
  if (frame.size() < 6) throw ProtocolError("short frame");
  uint32_t payload;
  std::memcpy(&payload, frame.data(), sizeof(payload));
  if (frame.size() - 4 < payload)
    throw ProtocolError("partial frame: need " + std::to_string(payload) + " bytes, have " +
                        std::to_string(frame.size() - 4));
  if (frame.size() - 4 > payload) throw ProtocolError("trailing bytes after the frame");
  Reader r(frame.data() + 4, payload);
  const uint8_t version = r.Get<uint8_t>();
  if (version != kProtocolVersion)
    throw ProtocolError("protocol version " + std::to_string(version) + ", expected " +
                        std::to_string(kProtocolVersion));
  const int t = r.Get<uint8_t>();
  if (!KnownType(t)) throw ProtocolError("unknown message type " + std::to_string(t));
  const std::string kinds = MessageSchema(t);
  std::vector<Field> out(kinds.size());
  for (size_t k = 0; k < kinds.size(); ++k) {
    Field& f = out[k];
    f.kind = FieldKind(kinds[k]);
    switch (f.kind) {
      case FieldKind::kI64: f.i = r.Get<int64_t>(); break;
      case FieldKind::kF64: f.f = r.Get<double>(); break;
      case FieldKind::kBool: f.i = r.Get<uint8_t>() ? 1 : 0; break;
      case FieldKind::kStr: {
        const uint32_t n = r.Get<uint32_t>();
        f.s.resize(n);
        r.Bytes(f.s.data(), n);
        break;
      }
      case FieldKind::kPairs: {
        const uint64_t n = r.Count(2 * sizeof(int64_t));
        f.a.resize(2 * n);
        r.Bytes(f.a.data(), 2 * n * sizeof(int64_t));
        break;
      }
      case FieldKind::kOptI64:
        f.present = r.Get<uint8_t>() != 0;
        if (f.present) f.i = r.Get<int64_t>();
        break;
      case FieldKind::kOptI64Array:
        f.present = r.Get<uint8_t>() != 0;
        if (!f.present) break;
        [[fallthrough]];
      case FieldKind::kI64Array: {
        const uint64_t n = r.Count(sizeof(int64_t));
        f.a.resize(n);
        r.Bytes(f.a.data(), n * sizeof(int64_t));
        break;
      }
      case FieldKind::kOptF32Array:
        f.present = r.Get<uint8_t>() != 0;
        if (f.present) {
          const uint64_t n = r.Count(sizeof(float));
          f.fa.resize(n);
          r.Bytes(f.fa.data(), n * sizeof(float));
        }
        break;
    }
  }
  if (!r.Done()) throw ProtocolError("trailing bytes inside the frame");
  *type = t;
  return out;
}

}  // namespace hcp::host
