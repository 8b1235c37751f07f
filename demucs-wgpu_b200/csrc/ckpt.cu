// torch.save checkpoints (`.th` / `.pth`) and the model kwargs of a checkpoint.
//
// A torch.save file is a zip (entries stored, not compressed) holding
// <root>/data.pkl — a pickle of the object graph — one raw blob per tensor
// storage under <root>/data/<key>, and <root>/byteorder (ckpt/mod.rs:1-10).
// The reader below walks the zip's central directory, runs the pickle opcodes
// torch.save emits (protocol 2: dicts, lists, tuples, ints, floats, strings,
// globals, REDUCE / BUILD / NEWOBJ, memo, persistent ids for storages), turns
// torch._utils._rebuild_tensor_v2 / _rebuild_parameter into tensor views and
// collections.OrderedDict into dicts, and leaves every other reduction opaque
// (ckpt/pickle.rs:123-560). The state dict is found as the reference finds it:
// under `model_state_dict`, `state_dict` or `state`, or the top-level dict
// itself (ckpt/mod.rs:244-275). Tensors are gathered through their strides
// and storage offsets into f32, with the dtype upcasts of the safetensors
// reader.
//
// The model kwargs (the safetensors `__metadata__["kwargs"]` JSON, or the
// pickled `kwargs` dict of a demucs `.th` package) are parsed and checked
// against the one architecture the kernels implement, the htdemucs default
// (config.rs:43-71, 150-215): a checkpoint of any other shape is rejected
// with the field that differs.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime.cuh"

namespace dmx {

namespace {

// ---------------------------------------------------------------------------
// zip (stored entries; zip64 sizes and offsets when present)
// ---------------------------------------------------------------------------
struct ZipEntry {
  uint64_t offset = 0;  // of the local file header
  uint64_t size = 0;
  int method = 0;
};

uint64_t rd(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = n - 1; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

std::map<std::string, ZipEntry> zip_directory(const uint8_t* z, size_t len) {
  auto bad = [](const std::string& m) { return Error(DMX_ERR_WEIGHTS, "checkpoint zip: " + m); };
  if (len < 22) throw bad("shorter than an end-of-directory record");
  size_t eocd = std::string::npos;
  for (size_t i = len - 22 + 1; i-- > 0 && len - i <= 22 + 65535;)
    if (rd(z + i, 4) == 0x06054b50u) {
      eocd = i;
      break;
    }
  if (eocd == std::string::npos) throw bad("no end-of-central-directory record");
  uint64_t count = rd(z + eocd + 10, 2), cd_size = rd(z + eocd + 12, 4), cd_off = rd(z + eocd + 16, 4);
  if ((count == 0xFFFF || cd_off == 0xFFFFFFFFu) && eocd >= 20 && rd(z + eocd - 20, 4) == 0x07064b50u) {
    const uint64_t z64 = rd(z + eocd - 20 + 8, 8);
    if (z64 + 56 > len || rd(z + z64, 4) != 0x06064b50u) throw bad("bad zip64 end record");
    count = rd(z + z64 + 32, 8);
    cd_size = rd(z + z64 + 40, 8);
    cd_off = rd(z + z64 + 48, 8);
  }
  if (cd_off > len || cd_size > len - cd_off) throw bad("central directory outside the file");
  std::map<std::string, ZipEntry> out;
  size_t p = cd_off;
  for (uint64_t i = 0; i < count; ++i) {
    if (p + 46 > len || rd(z + p, 4) != 0x02014b50u) throw bad("bad central directory entry");
    ZipEntry e;
    e.method = (int)rd(z + p + 10, 2);
    uint64_t csize = rd(z + p + 20, 4), usize = rd(z + p + 24, 4);
    const size_t nlen = rd(z + p + 28, 2), xlen = rd(z + p + 30, 2), clen = rd(z + p + 32, 2);
    e.offset = rd(z + p + 42, 4);
    if (p + 46 + nlen + xlen + clen > len) throw bad("central directory entry runs past the file");
    const std::string name(reinterpret_cast<const char*>(z + p + 46), nlen);
    // zip64 extended information: the 0xFFFFFFFF fields, in order
    for (size_t x = p + 46 + nlen; x + 4 <= p + 46 + nlen + xlen;) {
      const uint64_t id = rd(z + x, 2), sz = rd(z + x + 2, 2);
      if (id == 0x0001) {
        size_t q = x + 4;
        if (usize == 0xFFFFFFFFu) usize = rd(z + q, 8), q += 8;
        if (csize == 0xFFFFFFFFu) csize = rd(z + q, 8), q += 8;
        if (e.offset == 0xFFFFFFFFu) e.offset = rd(z + q, 8);
      }
      x += 4 + sz;
    }
    e.size = csize;
    if (e.method == 0 && csize != usize) throw bad(name + ": stored entry with mismatched sizes");
    out[name] = e;
    p += 46 + nlen + xlen + clen;
  }
  return out;
}

// The bytes of one stored entry.
std::pair<const uint8_t*, size_t> zip_read(const uint8_t* z, size_t len, const ZipEntry& e,
                                           const std::string& name) {
  if (e.method != 0)
    throw Error(DMX_ERR_WEIGHTS, "checkpoint zip: " + name + " is compressed (method " +
                                     std::to_string(e.method) + "); torch.save stores entries");
  if (e.offset + 30 > len || rd(z + e.offset, 4) != 0x04034b50u)
    throw Error(DMX_ERR_WEIGHTS, "checkpoint zip: bad local header for " + name);
  const uint64_t start = e.offset + 30 + rd(z + e.offset + 26, 2) + rd(z + e.offset + 28, 2);
  if (start > len || e.size > len - start)
    throw Error(DMX_ERR_WEIGHTS, "checkpoint zip: " + name + " runs past the file");
  return {z + start, (size_t)e.size};
}

// ---------------------------------------------------------------------------
// pickle
// ---------------------------------------------------------------------------
struct PValue;
using PV = std::shared_ptr<PValue>;

struct PValue {
  enum Kind { NONE, BOOL, INT, FLOAT, STR, BYTES, TUPLE, LIST, DICT, GLOBAL, STORAGE, TENSOR,
              FRACTION, OPAQUE } kind = NONE;
  int64_t i = 0;
  double f = 0.0;
  std::string s, s2;                       // STR / BYTES; GLOBAL module, name; STORAGE key, dtype
  std::vector<PV> items;                   // TUPLE / LIST
  std::vector<std::pair<PV, PV>> dict;     // DICT, in insertion order
  // STORAGE: numel in i; TENSOR: the storage, offset, size, stride
  PV storage;
  int64_t offset = 0;
  std::vector<int64_t> size, stride;
};

PV mk(PValue::Kind k) {
  auto v = std::make_shared<PValue>();
  v->kind = k;
  return v;
}

struct Unpickler {
  const uint8_t* p;
  const uint8_t* end;
  std::vector<PV> stack;
  std::vector<size_t> marks;
  std::map<uint64_t, PV> memo;

  [[noreturn]] void bad(const std::string& m) { throw Error(DMX_ERR_WEIGHTS, "checkpoint pickle: " + m); }
  const uint8_t* take(size_t n) {
    if ((size_t)(end - p) < n) bad("truncated");
    const uint8_t* q = p;
    p += n;
    return q;
  }
  uint64_t uint(int n) { return rd(take(n), n); }
  std::string line() {
    const uint8_t* q = p;
    while (p < end && *p != '\n') ++p;
    if (p >= end) bad("unterminated line");
    std::string s(reinterpret_cast<const char*>(q), p - q);
    ++p;
    return s;
  }
  PV pop() {
    if (stack.empty()) bad("stack underflow");
    PV v = stack.back();
    stack.pop_back();
    return v;
  }
  std::vector<PV> pop_mark() {
    if (marks.empty()) bad("no mark");
    const size_t m = marks.back();
    marks.pop_back();
    if (m > stack.size()) bad("mark past the stack");
    std::vector<PV> v(stack.begin() + m, stack.end());
    stack.resize(m);
    return v;
  }
  PV tuple(std::vector<PV> v) {
    PV t = mk(PValue::TUPLE);
    t->items = std::move(v);
    return t;
  }
  PV str(const std::string& s) {
    PV v = mk(PValue::STR);
    v->s = s;
    return v;
  }
  static bool is_global(const PV& v, const char* mod, const char* name) {
    return v && v->kind == PValue::GLOBAL && v->s == mod && v->s2 == name;
  }
  static int64_t as_int(const PV& v) {
    if (!v || (v->kind != PValue::INT && v->kind != PValue::BOOL))
      throw Error(DMX_ERR_WEIGHTS, "checkpoint pickle: expected an integer");
    return v->i;
  }
  static std::vector<int64_t> ints(const PV& v) {
    if (!v || (v->kind != PValue::TUPLE && v->kind != PValue::LIST))
      throw Error(DMX_ERR_WEIGHTS, "checkpoint pickle: expected a tuple of integers");
    std::vector<int64_t> out;
    for (const PV& x : v->items) out.push_back(as_int(x));
    return out;
  }

  // torch._utils._rebuild_tensor_v2(storage, offset, size, stride, ...) and the
  // parameter / OrderedDict / Fraction reductions; anything else is opaque
  PV reduce(const PV& fn, const PV& args) {
    const std::vector<PV>& a = args->items;
    if ((is_global(fn, "torch._utils", "_rebuild_tensor_v2") ||
         is_global(fn, "torch._utils", "_rebuild_tensor")) && a.size() >= 4) {
      if (!a[0] || a[0]->kind != PValue::STORAGE) bad("tensor without a storage");
      if (!a[1] || !a[2] || !a[3]) bad("tensor without its geometry");
      PV t = mk(PValue::TENSOR);
      t->storage = a[0];
      t->offset = as_int(a[1]);
      t->size = ints(a[2]);
      t->stride = ints(a[3]);
      if (t->size.size() != t->stride.size()) bad("tensor size and stride ranks differ");
      return t;
    }
    if (is_global(fn, "torch._utils", "_rebuild_parameter") && !a.empty()) return a[0];
    if (is_global(fn, "collections", "OrderedDict")) return mk(PValue::DICT);
    if (is_global(fn, "fractions", "Fraction")) {  // Fraction(num, den) or Fraction("num/den")
      PV v = mk(PValue::FRACTION);
      if (a.size() == 2 && a[0] && a[1]) {
        v->f = (double)as_int(a[0]) / (double)as_int(a[1]);
      } else if (a.size() == 1 && a[0] && a[0]->kind == PValue::STR) {
        const size_t slash = a[0]->s.find('/');
        const double num = std::strtod(a[0]->s.c_str(), nullptr);
        const double den =
            slash == std::string::npos ? 1.0 : std::strtod(a[0]->s.c_str() + slash + 1, nullptr);
        v->f = num / den;
      } else {
        return mk(PValue::OPAQUE);
      }
      return v;
    }
    return mk(PValue::OPAQUE);
  }

  // ('storage', <Storage class>, key, location, numel)
  PV persistent(const PV& pid) {
    if (!pid || pid->kind != PValue::TUPLE || pid->items.size() < 5) bad("unsupported persistent id");
    const PV& cls = pid->items[1];
    if (!cls || cls->kind != PValue::GLOBAL) bad("storage without a class");
    PV st = mk(PValue::STORAGE);
    st->s2 = cls->s2;  // FloatStorage, HalfStorage, ...
    const PV& key = pid->items[2];
    if (!key) bad("storage without a key");
    st->s = key->kind == PValue::STR ? key->s : std::to_string(key->i);
    st->i = as_int(pid->items[4]);
    return st;
  }

  PV run() {
    while (true) {
      const uint8_t op = *take(1);
      switch (op) {
        case 0x80: take(1); break;                                // PROTO
        case 0x95: take(8); break;                                // FRAME
        case '.': return pop();                                   // STOP
        case '(': marks.push_back(stack.size()); break;           // MARK
        case ')': stack.push_back(mk(PValue::TUPLE)); break;      // EMPTY_TUPLE
        case ']': stack.push_back(mk(PValue::LIST)); break;       // EMPTY_LIST
        case '}': stack.push_back(mk(PValue::DICT)); break;       // EMPTY_DICT
        case 'N': stack.push_back(mk(PValue::NONE)); break;       // NONE
        case 0x88: case 0x89: {                                   // NEWTRUE / NEWFALSE
          PV v = mk(PValue::BOOL);
          v->i = op == 0x88;
          stack.push_back(v);
          break;
        }
        case 'K': case 'M': case 'J': {                           // BININT1 / 2 / BININT
          PV v = mk(PValue::INT);
          v->i = op == 'K' ? (int64_t)uint(1) : op == 'M' ? (int64_t)uint(2) : (int64_t)(int32_t)uint(4);
          stack.push_back(v);
          break;
        }
        case 0x8a: {                                              // LONG1
          const size_t n = *take(1);
          if (n > 8) bad("integer wider than 64 bits");
          const uint8_t* b = take(n);
          uint64_t u = 0;
          for (size_t i = 0; i < n; ++i) u |= (uint64_t)b[i] << (8 * i);
          if (n > 0 && n < 8 && (b[n - 1] & 0x80)) u |= ~0ull << (8 * n);  // sign extend
          PV v = mk(PValue::INT);
          v->i = (int64_t)u;
          stack.push_back(v);
          break;
        }
        case 'I': {                                               // INT (text)
          const std::string s = line();
          PV v = mk(s == "00" || s == "01" ? PValue::BOOL : PValue::INT);
          v->i = std::strtoll(s.c_str(), nullptr, 10);
          stack.push_back(v);
          break;
        }
        case 'G': {                                               // BINFLOAT (big endian)
          const uint8_t* b = take(8);
          uint64_t u = 0;
          for (int i = 0; i < 8; ++i) u = (u << 8) | b[i];
          PV v = mk(PValue::FLOAT);
          std::memcpy(&v->f, &u, 8);
          stack.push_back(v);
          break;
        }
        case 'X': case 0x8c: case 'B': case 'C': case 0x8e: {     // unicode / bytes
          const size_t n = op == 0x8c || op == 'C' ? uint(1) : op == 0x8e ? uint(8) : uint(4);
          const uint8_t* b = take(n);
          PV v = mk(op == 'X' || op == 0x8c ? PValue::STR : PValue::BYTES);
          v->s.assign(reinterpret_cast<const char*>(b), n);
          stack.push_back(v);
          break;
        }
        case 'c': {                                               // GLOBAL module\nname\n
          PV g = mk(PValue::GLOBAL);
          g->s = line();
          g->s2 = line();
          stack.push_back(g);
          break;
        }
        case 0x93: {                                              // STACK_GLOBAL
          PV name = pop(), mod = pop();
          PV g = mk(PValue::GLOBAL);
          g->s = mod->s;
          g->s2 = name->s;
          stack.push_back(g);
          break;
        }
        case 't': stack.push_back(tuple(pop_mark())); break;      // TUPLE
        case 0x85: case 0x86: case 0x87: {                        // TUPLE1..3
          const size_t n = op - 0x84;
          if (stack.size() < n) bad("stack underflow");
          std::vector<PV> v(stack.end() - n, stack.end());
          stack.resize(stack.size() - n);
          stack.push_back(tuple(std::move(v)));
          break;
        }
        case 'l': {                                               // LIST
          PV l = mk(PValue::LIST);
          l->items = pop_mark();
          stack.push_back(l);
          break;
        }
        case 'd': {                                               // DICT
          PV d = mk(PValue::DICT);
          std::vector<PV> v = pop_mark();
          if (v.size() % 2) bad("odd dict items");
          for (size_t i = 0; i < v.size(); i += 2) d->dict.push_back({v[i], v[i + 1]});
          stack.push_back(d);
          break;
        }
        case 'a': {                                               // APPEND
          PV x = pop();
          if (stack.empty() || stack.back()->kind != PValue::LIST) bad("append to a non-list");
          stack.back()->items.push_back(x);
          break;
        }
        case 'e': {                                               // APPENDS
          std::vector<PV> v = pop_mark();
          if (stack.empty()) bad("appends to nothing");
          if (stack.back()->kind == PValue::LIST)
            for (PV& x : v) stack.back()->items.push_back(x);
          break;
        }
        case 's': {                                               // SETITEM
          PV v = pop(), k = pop();
          if (stack.empty()) bad("setitem on nothing");
          if (stack.back()->kind == PValue::DICT) stack.back()->dict.push_back({k, v});
          break;
        }
        case 'u': {                                               // SETITEMS
          std::vector<PV> v = pop_mark();
          if (v.size() % 2 || stack.empty()) bad("bad setitems");
          if (stack.back()->kind == PValue::DICT)
            for (size_t i = 0; i < v.size(); i += 2) stack.back()->dict.push_back({v[i], v[i + 1]});
          break;
        }
        case 'q': memo[uint(1)] = stack.empty() ? nullptr : stack.back(); break;  // BINPUT
        case 'r': memo[uint(4)] = stack.empty() ? nullptr : stack.back(); break;  // LONG_BINPUT
        case 0x94: memo[memo.size()] = stack.empty() ? nullptr : stack.back(); break;  // MEMOIZE
        case 'h': case 'j': {                                     // BINGET / LONG_BINGET
          auto it = memo.find(uint(op == 'h' ? 1 : 4));
          if (it == memo.end()) bad("memo miss");
          stack.push_back(it->second);
          break;
        }
        case 'p': memo[std::strtoull(line().c_str(), nullptr, 10)] = stack.empty() ? nullptr : stack.back(); break;
        case 'g': {
          auto it = memo.find(std::strtoull(line().c_str(), nullptr, 10));
          if (it == memo.end()) bad("memo miss");
          stack.push_back(it->second);
          break;
        }
        case 'R': {                                               // REDUCE
          PV args = pop(), fn = pop();
          if (!args || args->kind != PValue::TUPLE) bad("reduce without an argument tuple");
          stack.push_back(reduce(fn, args));
          break;
        }
        case 0x81: {                                              // NEWOBJ
          pop();
          pop();
          stack.push_back(mk(PValue::OPAQUE));
          break;
        }
        case 'b': pop(); break;                                   // BUILD: state ignored
        case 'Q': stack.push_back(persistent(pop())); break;      // BINPERSID
        case '0': pop(); break;                                   // POP
        case '2': stack.push_back(stack.empty() ? nullptr : stack.back()); break;  // DUP
        case '1': pop_mark(); break;                              // POP_MARK
        default: {
          char m[64];
          snprintf(m, sizeof(m), "unsupported opcode 0x%02x", op);
          bad(m);
        }
      }
    }
  }
};

// Storage dtype (legacy typed-storage class name) -> element width and decoder
// name of the safetensors reader.
std::pair<int, const char*> storage_dtype(const std::string& cls) {
  if (cls == "FloatStorage") return {4, "F32"};
  if (cls == "HalfStorage") return {2, "F16"};
  if (cls == "BFloat16Storage") return {2, "BF16"};
  if (cls == "DoubleStorage") return {8, "F64"};
  if (cls == "LongStorage") return {8, "I64"};
  if (cls == "IntStorage") return {4, "I32"};
  if (cls == "ShortStorage") return {2, "I16"};
  if (cls == "CharStorage") return {1, "I8"};
  if (cls == "ByteStorage") return {1, "U8"};
  if (cls == "BoolStorage") return {1, "BOOL"};
  return {0, nullptr};
}

const PValue* dict_get(const PValue& d, const char* key) {
  for (const auto& kv : d.dict)
    if (kv.first && kv.first->kind == PValue::STR && kv.first->s == key) return kv.second.get();
  return nullptr;
}

bool has_tensor(const PValue& d) {
  for (const auto& kv : d.dict)
    if (kv.second && kv.second->kind == PValue::TENSOR) return true;
  return false;
}

// ---------------------------------------------------------------------------
// kwargs: a small JSON reader (numbers, strings, booleans, arrays, objects)
// ---------------------------------------------------------------------------
struct JValue {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double n = 0.0;
  bool b = false;
  std::string s;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;
  const JValue* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  [[noreturn]] void bad() { throw Error(DMX_ERR_WEIGHTS, "checkpoint kwargs are not valid JSON"); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  JValue value() {
    ws();
    if (p >= end) bad();
    JValue v;
    if (*p == '{') {
      v.kind = JValue::OBJ;
      ++p;
      ws();
      if (p < end && *p == '}') return ++p, v;
      while (true) {
        ws();
        JValue k = value();
        if (k.kind != JValue::STR) bad();
        ws();
        if (p >= end || *p++ != ':') bad();
        v.obj.push_back({k.s, value()});
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') return ++p, v;
        bad();
      }
    }
    if (*p == '[') {
      v.kind = JValue::ARR;
      ++p;
      ws();
      if (p < end && *p == ']') return ++p, v;
      while (true) {
        v.arr.push_back(value());
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') return ++p, v;
        bad();
      }
    }
    if (*p == '"') {
      v.kind = JValue::STR;
      ++p;
      while (p < end && *p != '"') {
        if (*p == '\\' && p + 1 < end) ++p;
        v.s += *p++;
      }
      if (p >= end) bad();
      ++p;
      return v;
    }
    if (end - p >= 4 && !std::strncmp(p, "true", 4)) return p += 4, v.kind = JValue::BOOL, v.b = true, v;
    if (end - p >= 5 && !std::strncmp(p, "false", 5)) return p += 5, v.kind = JValue::BOOL, v;
    if (end - p >= 4 && !std::strncmp(p, "null", 4)) return p += 4, v;
    char* e = nullptr;
    v.kind = JValue::NUM;
    v.n = std::strtod(p, &e);
    if (e == p) bad();
    p = e;
    return v;
  }
};

// The htdemucs default (config.rs:43-71): the architecture these kernels implement.
struct Expect {
  const char* name;
  double value;
};
const Expect kArch[] = {
    {"audio_channels", 2}, {"samplerate", 44100}, {"channels", 48}, {"growth", 2},
    {"nfft", 4096}, {"depth", 4}, {"stride", 4}, {"kernel_size", 8}, {"context", 1},
    {"freq_emb", 0.2}, {"emb_scale", 10}, {"bottom_channels", 512}, {"t_layers", 5},
    {"t_heads", 8}, {"t_hidden_scale", 4}, {"t_max_period", 10000}, {"t_weight_pos_embed", 1}};

void check_field(const char* name, double got, double want) {
  if (!(std::fabs(got - want) <= 1e-9 * std::max(1.0, std::fabs(want)))) {
    char m[256];
    snprintf(m, sizeof(m),
             "checkpoint kwargs: %s = %g, but this backend implements the htdemucs default %g",
             name, got, want);
    throw Error(DMX_ERR_INVALID, m);
  }
}

void check_sources(size_t n) {
  if (n != 4)
    throw Error(DMX_ERR_INVALID, "checkpoint kwargs: " + std::to_string(n) +
                                     " sources, but this backend implements the htdemucs default 4");
}

}  // namespace

void check_kwargs_json(const std::string& text) {
  JParser jp{text.data(), text.data() + text.size()};
  const JValue v = jp.value();
  if (v.kind != JValue::OBJ) throw Error(DMX_ERR_WEIGHTS, "checkpoint kwargs are not a JSON object");
  for (const Expect& e : kArch) {
    const JValue* f = v.get(e.name);
    if (f && f->kind == JValue::NUM) check_field(e.name, f->n, e.value);
  }
  if (const JValue* c = v.get("cac"))
    if (c->kind == JValue::BOOL && !c->b) throw Error(DMX_ERR_INVALID, "checkpoint kwargs: cac = false, but this backend implements complex-as-channels");
  if (const JValue* s = v.get("sources"))
    if (s->kind == JValue::ARR) check_sources(s->arr.size());
  if (const JValue* seg = v.get("segment")) {  // a number, or a Fraction object
    double val = NAN;
    if (seg->kind == JValue::NUM) val = seg->n;
    if (seg->kind == JValue::OBJ && seg->get("numerator") && seg->get("denominator"))
      val = seg->get("numerator")->n / seg->get("denominator")->n;
    if (!std::isnan(val)) check_field("segment", val, 39.0 / 5.0);
  }
}

bool is_torch_zip(const void* blob, size_t len) {
  return len >= 4 && rd(static_cast<const uint8_t*>(blob), 4) == 0x04034b50u;
}

std::map<std::string, HostTensor> parse_torch_zip(const void* blob, size_t len) {
  const uint8_t* z = static_cast<const uint8_t*>(blob);
  const auto dir = zip_directory(z, len);
  std::string root;
  for (const auto& kv : dir) {
    const std::string& n = kv.first;
    if (n.size() >= 9 && n.compare(n.size() - 9, 9, "/data.pkl") == 0) {
      root = n.substr(0, n.size() - 9);
      break;
    }
  }
  if (root.empty() && !dir.count("data.pkl"))
    throw Error(DMX_ERR_WEIGHTS, "checkpoint zip holds no <root>/data.pkl: not a torch.save file");
  const std::string pre = root.empty() ? "" : root + "/";
  bool big_endian = false;
  if (dir.count(pre + "byteorder")) {
    const auto bo = zip_read(z, len, dir.at(pre + "byteorder"), "byteorder");
    big_endian = std::string(reinterpret_cast<const char*>(bo.first), bo.second).find("big") == 0;
  }
  const auto pkl = zip_read(z, len, dir.at(pre + "data.pkl"), "data.pkl");
  Unpickler up{pkl.first, pkl.first + pkl.second, {}, {}, {}};
  const PV top = up.run();
  if (!top || top->kind != PValue::DICT) throw Error(DMX_ERR_WEIGHTS, "checkpoint top level is not a dict");
  const PValue* state = nullptr;
  for (const char* key : {"model_state_dict", "state_dict", "state"}) {
    const PValue* d = dict_get(*top, key);
    if (d && d->kind == PValue::DICT && has_tensor(*d)) {
      state = d;
      break;
    }
  }
  if (!state && has_tensor(*top)) state = top.get();
  if (!state)
    throw Error(DMX_ERR_WEIGHTS, "checkpoint has no tensor state dict (looked for "
                                 "model_state_dict / state_dict / state)");
  // the demucs package's pickled kwargs, checked like the safetensors JSON
  if (const PValue* kw = dict_get(*top, "kwargs"))
    if (kw->kind == PValue::DICT) {
      for (const Expect& e : kArch) {
        const PValue* f = dict_get(*kw, e.name);
        if (f && (f->kind == PValue::INT || f->kind == PValue::FLOAT))
          check_field(e.name, f->kind == PValue::INT ? (double)f->i : f->f, e.value);
      }
      if (const PValue* s = dict_get(*kw, "sources"))
        if (s->kind == PValue::LIST || s->kind == PValue::TUPLE) check_sources(s->items.size());
      if (const PValue* seg = dict_get(*kw, "segment"))
        if (seg->kind == PValue::FRACTION || seg->kind == PValue::FLOAT || seg->kind == PValue::INT)
          check_field("segment", seg->kind == PValue::INT ? (double)seg->i : seg->f, 39.0 / 5.0);
    }
  std::map<std::string, HostTensor> out;
  for (const auto& kv : state->dict) {
    if (!kv.first || kv.first->kind != PValue::STR || !kv.second) continue;
    const PValue& t = *kv.second;
    if (t.kind == PValue::NONE || t.kind == PValue::OPAQUE) continue;
    const std::string& name = kv.first->s;
    if (t.kind != PValue::TENSOR) throw Error(DMX_ERR_WEIGHTS, "state dict entry " + name + " is not a tensor");
    const PValue& st = *t.storage;
    const auto dt = storage_dtype(st.s2);
    if (!dt.second) throw Error(DMX_ERR_WEIGHTS, name + ": unsupported storage " + st.s2);
    const std::string entry = pre + "data/" + st.s;
    if (!dir.count(entry)) throw Error(DMX_ERR_WEIGHTS, "missing storage entry " + entry);
    const auto raw = zip_read(z, len, dir.at(entry), entry);
    const size_t avail = raw.second / dt.first;
    // the element of every index of the view: offset + sum index * stride
    size_t count = 1;
    for (int64_t d : t.size) {
      if (d < 0) throw Error(DMX_ERR_WEIGHTS, name + ": negative size");
      count *= (size_t)d;
    }
    int64_t lo = t.offset, hi = t.offset;
    for (size_t d = 0; d < t.size.size(); ++d)
      if (t.size[d] > 0) {
        const int64_t span = (t.size[d] - 1) * t.stride[d];
        if (span < 0) lo += span; else hi += span;
      }
    if (count > 0 && (lo < 0 || (size_t)hi >= avail))
      throw Error(DMX_ERR_WEIGHTS, name + ": view runs past its storage");
    std::vector<uint8_t> bytes(count * dt.first);
    std::vector<int64_t> idx(t.size.size(), 0);
    for (size_t e = 0; e < count; ++e) {
      int64_t at = t.offset;
      for (size_t d = 0; d < idx.size(); ++d) at += idx[d] * t.stride[d];
      const uint8_t* src = raw.first + (size_t)at * dt.first;
      uint8_t* dst = bytes.data() + e * dt.first;
      for (int b = 0; b < dt.first; ++b) dst[b] = big_endian ? src[dt.first - 1 - b] : src[b];
      for (size_t d = idx.size(); d-- > 0;) {
        if (++idx[d] < t.size[d]) break;
        idx[d] = 0;
      }
    }
    HostTensor h;
    h.shape = t.size;
    h.owned = std::make_shared<std::vector<float>>(
        std::string(dt.second) == "F32" ? std::vector<float>(count)
                                        : decode_tensor(reinterpret_cast<const char*>(bytes.data()),
                                                        count, dt.second));
    if (std::string(dt.second) == "F32") std::memcpy(h.owned->data(), bytes.data(), count * 4);
    h.data = h.owned->data();
    out[name] = h;
  }
  return out;
}

std::map<std::string, HostTensor> parse_checkpoint(const void* blob, size_t len) {
  if (!blob) throw Error(DMX_ERR_INVALID, "checkpoint blob is NULL");
  return is_torch_zip(blob, len) ? parse_torch_zip(blob, len) : parse_safetensors(blob, len);
}

}  // namespace dmx
