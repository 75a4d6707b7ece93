// N-API addon "h2cuda.node": the Node.js binding of libh2cuda (include/h2cuda.h) for the reference engine's
// JavaScript host. cuda.js (next to this file) builds the backend object of cpu.js:52-68 on top of it.
//
// UNVERIFIED: this build image has no Node.js and no node-addon-api headers, so this file is compiled and run
// nowhere here. The same C ABI is exercised by the Python binding (_lib.py, backend.py) and its tests.
//
// The addon owns nothing but the engine handle (a Napi::External). forward / forwardBatch run on a libuv worker
// thread (Napi::AsyncWorker) and resolve a Promise, so the event loop never blocks while the GPU computes: the
// reference gets the same property from its leader Worker (cpu-worker.js:1-7). Calls on one engine are serialised
// by the JavaScript caller, as cpu.js keeps a single outstanding request (cpu.js:33-50).
#include <napi.h>

#include <cstring>
#include <string>
#include <vector>

#include "h2cuda.h"

namespace {

h2c_engine* engine_of(const Napi::Value& v) { return v.As<Napi::External<h2c_engine>>().Data(); }

// status -> exception; "context full" keeps the reference's message (cpu-worker.js:173)
void check(Napi::Env env, h2c_engine* e, int rc) {
  if (rc == H2C_ERR_CONTEXT_FULL) throw Napi::Error::New(env, "context full");
  if (rc != H2C_OK) throw Napi::Error::New(env, h2c_last_error(e));
}

std::vector<int32_t> ints(const Napi::Value& v) {
  auto a = v.As<Napi::Int32Array>();
  return std::vector<int32_t>(a.Data(), a.Data() + a.ElementLength());
}

int32_t field(const Napi::Object& o, const char* k) { return o.Get(k).As<Napi::Number>().Int32Value(); }

h2c_config config_of(const Napi::Object& o) {
  h2c_config c{};
  c.dim = field(o, "dim");
  c.layers = field(o, "layers");
  c.ffn = field(o, "ffn");
  c.heads = field(o, "heads");
  c.kv_heads = field(o, "kv_heads");
  c.vocab = field(o, "vocab");
  c.ctx = field(o, "ctx");
  c.max_chunk = field(o, "max_chunk");
  c.max_seqs = field(o, "max_seqs");
  c.eps = o.Get("eps").As<Napi::Number>().FloatValue();
  c.rope_theta = o.Get("rope_theta").As<Napi::Number>().DoubleValue();
  return c;
}

// h2c.tpUniqueId() -> Buffer(H2C_TP_ID_BYTES): a tensor-parallel group's id, created by rank 0 and handed to the
// other ranks' processes by the host (e.g. over the page's or the server's own channel)
Napi::Value TpUniqueId(const Napi::CallbackInfo& info) {
  Napi::Env env = info.Env();
  auto buf = Napi::Buffer<uint8_t>::New(env, H2C_TP_ID_BYTES);
  check(env, nullptr, h2c_tp_unique_id(buf.Data()));
  return buf;
}

// h2c.createTp(device, cfg, world, rank, Buffer id, timeoutMs): one rank of a tensor-parallel group (every rank then
// loads the same full tensors and makes the same calls)
Napi::Value CreateTp(const Napi::CallbackInfo& info) {
  Napi::Env env = info.Env();
  const h2c_config c = config_of(info[1].As<Napi::Object>());
  auto id = info[4].As<Napi::Buffer<uint8_t>>();
  if (id.Length() != H2C_TP_ID_BYTES) throw Napi::Error::New(env, "tensor-parallel id has the wrong length");
  h2c_engine* e = nullptr;
  check(env, nullptr, h2c_create_tp(info[0].As<Napi::Number>().Int32Value(), &c, info[2].As<Napi::Number>().Int32Value(),
                                    info[3].As<Napi::Number>().Int32Value(), id.Data(),
                                    info[5].As<Napi::Number>().Int32Value(), &e));
  return Napi::External<h2c_engine>::New(env, e);
}

// h2c.create(device, {dim, layers, ffn, heads, kv_heads, vocab, ctx, max_chunk, max_seqs, eps, rope_theta})
Napi::Value Create(const Napi::CallbackInfo& info) {
  Napi::Env env = info.Env();
  const h2c_config c = config_of(info[1].As<Napi::Object>());
  h2c_engine* e = nullptr;
  check(env, nullptr, h2c_create(info[0].As<Napi::Number>().Int32Value(), &c, &e));
  return Napi::External<h2c_engine>::New(env, e);
}

// h2c.setTensor(engine, kind, layer, ggmlType, ArrayBuffer bytes, offset, nbytes): raw GGUF blocks, copied once
Napi::Value SetTensor(const Napi::CallbackInfo& info) {
  h2c_engine* e = engine_of(info[0]);
  auto buf = info[4].As<Napi::ArrayBuffer>();
  const uint8_t* p = static_cast<const uint8_t*>(buf.Data()) + info[5].As<Napi::Number>().Int64Value();
  check(info.Env(), e,
        h2c_set_tensor(e, info[1].As<Napi::Number>().Int32Value(), info[2].As<Napi::Number>().Int32Value(),
                       info[3].As<Napi::Number>().Int32Value(), p, (uint64_t)info[6].As<Napi::Number>().Int64Value()));
  return info.Env().Undefined();
}

// h2c.setTensorConcat(engine, kind, layer, ArrayBuffer bytes, [{type, offset, nbytes}, ...]): the rows of several
// GGUF tensors of one type concatenated ([q;k;v], [gate;up], [bq;bk;bv]), as cpu-worker.js:57-63, 106-122 does
Napi::Value SetTensorConcat(const Napi::CallbackInfo& info) {
  h2c_engine* e = engine_of(info[0]);
  auto buf = info[3].As<Napi::ArrayBuffer>();
  const uint8_t* base = static_cast<const uint8_t*>(buf.Data());
  auto parts = info[4].As<Napi::Array>();
  std::vector<uint8_t> joined;
  int type = -1;
  for (uint32_t i = 0; i < parts.Length(); i++) {
    const Napi::Object t = parts.Get(i).As<Napi::Object>();
    const int ty = t.Get("type").As<Napi::Number>().Int32Value();
    if (type >= 0 && ty != type) throw Napi::Error::New(info.Env(), "setTensorConcat: tensors of different types");
    type = ty;
    const int64_t off = t.Get("offset").As<Napi::Number>().Int64Value();
    const int64_t n = t.Get("nbytes").As<Napi::Number>().Int64Value();
    joined.insert(joined.end(), base + off, base + off + n);
  }
  check(info.Env(), e,
        h2c_set_tensor(e, info[1].As<Napi::Number>().Int32Value(), info[2].As<Napi::Number>().Int32Value(), type,
                       joined.data(), joined.size()));
  return info.Env().Undefined();
}

class ForwardWorker : public Napi::AsyncWorker {
 public:
  ForwardWorker(Napi::Env env, h2c_engine* e, int seq, std::vector<int32_t> ids, int pos, double temp, uint32_t seed)
      : Napi::AsyncWorker(env), e_(e), seq_(seq), ids_(std::move(ids)), pos_(pos), temp_(temp), seed_(seed),
        deferred_(Napi::Promise::Deferred::New(env)) {}
  void Execute() override {
    const int rc = h2c_forward(e_, seq_, ids_.data(), (int32_t)ids_.size(), pos_, temp_, seed_, &next_);
    if (rc != H2C_OK) SetError(rc == H2C_ERR_CONTEXT_FULL ? "context full" : h2c_last_error(e_));
  }
  void OnOK() override { deferred_.Resolve(Napi::Number::New(Env(), next_)); }
  void OnError(const Napi::Error& err) override { deferred_.Reject(err.Value()); }
  Napi::Promise Promise() { return deferred_.Promise(); }

 private:
  h2c_engine* e_;
  int seq_;
  std::vector<int32_t> ids_;
  int pos_;
  double temp_;
  uint32_t seed_;
  int32_t next_ = 0;
  Napi::Promise::Deferred deferred_;
};

// h2c.forward(engine, seq, Int32Array ids, pos, temperature, seed) -> Promise<int next>
Napi::Value Forward(const Napi::CallbackInfo& info) {
  auto* w = new ForwardWorker(info.Env(), engine_of(info[0]), info[1].As<Napi::Number>().Int32Value(), ints(info[2]),
                              info[3].As<Napi::Number>().Int32Value(), info[4].As<Napi::Number>().DoubleValue(),
                              info[5].As<Napi::Number>().Uint32Value());
  w->Queue();
  return w->Promise();
}

class ForwardBatchWorker : public Napi::AsyncWorker {
 public:
  ForwardBatchWorker(Napi::Env env, h2c_engine* e, std::vector<int32_t> s, std::vector<int32_t> i,
                     std::vector<int32_t> p, double temp, uint32_t seed)
      : Napi::AsyncWorker(env), e_(e), s_(std::move(s)), i_(std::move(i)), p_(std::move(p)), temp_(temp),
        seed_(seed), next_(s_.size()), deferred_(Napi::Promise::Deferred::New(env)) {}
  void Execute() override {
    if (i_.size() != s_.size() || p_.size() != s_.size()) return SetError("seqs, ids and pos differ in length");
    const int rc = h2c_forward_batch(e_, (int32_t)s_.size(), s_.data(), i_.data(), p_.data(), temp_, seed_, next_.data());
    if (rc != H2C_OK) SetError(rc == H2C_ERR_CONTEXT_FULL ? "context full" : h2c_last_error(e_));
  }
  void OnOK() override {
    auto out = Napi::Int32Array::New(Env(), next_.size());
    for (size_t k = 0; k < next_.size(); k++) out[k] = next_[k];
    deferred_.Resolve(out);
  }
  void OnError(const Napi::Error& err) override { deferred_.Reject(err.Value()); }
  Napi::Promise Promise() { return deferred_.Promise(); }

 private:
  h2c_engine* e_;
  std::vector<int32_t> s_, i_, p_;
  double temp_;
  uint32_t seed_;
  std::vector<int32_t> next_;
  Napi::Promise::Deferred deferred_;
};

// h2c.forwardBatch(engine, Int32Array seqs, Int32Array ids, Int32Array pos, temperature, seed) -> Promise<Int32Array>
Napi::Value ForwardBatch(const Napi::CallbackInfo& info) {
  auto* w = new ForwardBatchWorker(info.Env(), engine_of(info[0]), ints(info[1]), ints(info[2]), ints(info[3]),
                                   info[4].As<Napi::Number>().DoubleValue(), info[5].As<Napi::Number>().Uint32Value());
  w->Queue();
  return w->Promise();
}

// h2c.readLogits(engine, seq, vocab) -> Float32Array(vocab)
Napi::Value ReadLogits(const Napi::CallbackInfo& info) {
  h2c_engine* e = engine_of(info[0]);
  const int vocab = info[2].As<Napi::Number>().Int32Value();
  auto out = Napi::Float32Array::New(info.Env(), vocab);
  check(info.Env(), e, h2c_read_logits(e, info[1].As<Napi::Number>().Int32Value(), out.Data(), vocab));
  return out;
}

// h2c.profile(engine, seq, Int32Array ids, pos) -> {op name: ms} (the reference's profile names, cpu-worker.js:32)
Napi::Value Profile(const Napi::CallbackInfo& info) {
  static const char* kNames[H2C_NPROF] = {"embed",    "norm+quantize", "matvec qkv",     "rope+kv",
                                          "attention", "quantize",     "matvec o",       "matvec gate+up",
                                          "swiglu+quantize", "matvec down", "matvec output"};
  h2c_engine* e = engine_of(info[0]);
  std::vector<int32_t> ids = ints(info[2]);
  double ms[H2C_NPROF];
  check(info.Env(), e, h2c_profile(e, info[1].As<Napi::Number>().Int32Value(), ids.data(), (int32_t)ids.size(),
                                   info[3].As<Napi::Number>().Int32Value(), ms));
  Napi::Object o = Napi::Object::New(info.Env());
  for (int k = 0; k < H2C_NPROF; k++) o.Set(kNames[k], Napi::Number::New(info.Env(), ms[k]));
  return o;
}

Napi::Value DeviceBytes(const Napi::CallbackInfo& info) {
  return Napi::Number::New(info.Env(), (double)h2c_device_bytes(engine_of(info[0])));
}

Napi::Value Destroy(const Napi::CallbackInfo& info) {
  h2c_destroy(engine_of(info[0]));
  return info.Env().Undefined();
}

Napi::Object Init(Napi::Env env, Napi::Object exports) {
  exports.Set("create", Napi::Function::New(env, Create));
  exports.Set("tpUniqueId", Napi::Function::New(env, TpUniqueId));
  exports.Set("createTp", Napi::Function::New(env, CreateTp));
  exports.Set("setTensor", Napi::Function::New(env, SetTensor));
  exports.Set("setTensorConcat", Napi::Function::New(env, SetTensorConcat));
  exports.Set("forward", Napi::Function::New(env, Forward));
  exports.Set("forwardBatch", Napi::Function::New(env, ForwardBatch));
  exports.Set("readLogits", Napi::Function::New(env, ReadLogits));
  exports.Set("profile", Napi::Function::New(env, Profile));
  exports.Set("deviceBytes", Napi::Function::New(env, DeviceBytes));
  exports.Set("destroy", Napi::Function::New(env, Destroy));
  return exports;
}

}  // namespace

NODE_API_MODULE(h2cuda, Init)
