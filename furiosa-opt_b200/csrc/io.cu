// Host I/O: safetensors files streamed straight into device storages.
//
// The reference loads a tensor with `HostTensor::from_safetensors(view)` and uploads it with
// `to_hbm` (furiosa-opt-std/src/tensor/memory.rs:197-222): the view's shape must equal the Element
// mapping's pair-split sizes (`flat_shape`) and its little-endian bytes are the packed device image
// as they are. Here the file's header is parsed once (the safetensors layout: an 8-byte
// little-endian header length, a JSON object of {name: {dtype, shape, data_offsets}}, then the
// data), and a tensor's bytes move file -> pinned staging -> device in chunks, the read of one chunk
// overlapping the copy of the previous one.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "ctx.hpp"

struct fopt_safetensors {
  struct Entry {
    std::string name, dtype;
    std::vector<int64_t> shape;
    int64_t begin = 0, end = 0;  // byte offsets into the data region
  };
  std::string path;
  int64_t data_start = 0, file_size = 0;
  std::vector<Entry> entries;
};

namespace fopt {
namespace {

// A small JSON reader for the safetensors header: objects, arrays, strings, integers, literals.
struct Json {
  const std::string& s;
  size_t i = 0;
  explicit Json(const std::string& text) : s(text) {}
  [[noreturn]] void fail(const char* what) const {
    throw Fail{FOPT_ERR_INVALID, std::string("safetensors header: ") + what + " at byte " + std::to_string(i)};
  }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool eat(char c) {
    ws();
    if (i < s.size() && s[i] == c) {
      ++i;
      return true;
    }
    return false;
  }
  void expect(char c) {
    if (!eat(c)) fail("unexpected character");
  }
  std::string str() {
    ws();
    if (i >= s.size() || s[i] != '"') fail("expected a string");
    ++i;
    std::string out;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) fail("bad escape");
        char e = s[i++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {  // code point -> UTF-8 (names are ASCII in practice)
            if (i + 4 > s.size()) fail("bad \\u escape");
            unsigned cp = (unsigned)std::stoul(s.substr(i, 4), nullptr, 16);
            i += 4;
            if (cp < 0x80) {
              out += (char)cp;
            } else if (cp < 0x800) {
              out += (char)(0xC0 | (cp >> 6));
              out += (char)(0x80 | (cp & 0x3F));
            } else {
              out += (char)(0xE0 | (cp >> 12));
              out += (char)(0x80 | ((cp >> 6) & 0x3F));
              out += (char)(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i >= s.size()) fail("unterminated string");
    ++i;
    return out;
  }
  int64_t integer() {
    ws();
    size_t j = i;
    if (j < s.size() && s[j] == '-') ++j;
    while (j < s.size() && s[j] >= '0' && s[j] <= '9') ++j;
    if (j == i) fail("expected an integer");
    int64_t v = std::stoll(s.substr(i, j - i));
    i = j;
    return v;
  }
  void skip() {  // any value
    ws();
    if (i >= s.size()) fail("truncated");
    char c = s[i];
    if (c == '{') {
      ++i;
      if (eat('}')) return;
      do {
        str();
        expect(':');
        skip();
      } while (eat(','));
      expect('}');
    } else if (c == '[') {
      ++i;
      if (eat(']')) return;
      do skip();
      while (eat(','));
      expect(']');
    } else if (c == '"') {
      str();
    } else {
      while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
    }
  }
};

void parse_header(const std::string& text, fopt_safetensors& st) {
  Json j(text);
  j.expect('{');
  if (j.eat('}')) return;
  do {
    std::string name = j.str();
    j.expect(':');
    if (name == "__metadata__") {
      j.skip();
      continue;
    }
    fopt_safetensors::Entry e;
    e.name = name;
    bool have_dtype = false, have_shape = false, have_off = false;
    j.expect('{');
    if (!j.eat('}')) {
      do {
        std::string key = j.str();
        j.expect(':');
        if (key == "dtype") {
          e.dtype = j.str();
          have_dtype = true;
        } else if (key == "shape") {
          j.expect('[');
          if (!j.eat(']')) {
            do e.shape.push_back(j.integer());
            while (j.eat(','));
            j.expect(']');
          }
          have_shape = true;
        } else if (key == "data_offsets") {
          j.expect('[');
          e.begin = j.integer();
          j.expect(',');
          e.end = j.integer();
          j.expect(']');
          have_off = true;
        } else {
          j.skip();
        }
      } while (j.eat(','));
      j.expect('}');
    }
    if (!have_dtype || !have_shape || !have_off || e.begin < 0 || e.end < e.begin)
      throw Fail{FOPT_ERR_INVALID, "safetensors header: incomplete entry " + name};
    st.entries.push_back(std::move(e));
  } while (j.eat(','));
  j.expect('}');
}

// `flat_shape` of memory.rs:201-209: pairs split recursively, any other node is one dimension.
void flat_shape(const Node& n, std::vector<int64_t>& out) {
  if (n.kind == Node::Pair) {
    flat_shape(*n.a, out);
    flat_shape(*n.b, out);
  } else {
    out.push_back(n.size);
  }
}

constexpr size_t kChunk = 8u << 20;  // pinned staging: two 8 MiB buffers per context

}  // namespace
}  // namespace fopt

using namespace fopt;

extern "C" {

fopt_status fopt_st_open(const char* path, fopt_safetensors** out) {
  if (!path || !out) return FOPT_ERR_INVALID;
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    g_noctx_err = std::string("fopt_st_open: cannot open ") + path;
    return FOPT_ERR_INVALID;
  }
  auto st = new fopt_safetensors;
  st->path = path;
  try {
    unsigned char len8[8];
    if (fread(len8, 1, 8, f) != 8) throw Fail{FOPT_ERR_INVALID, "safetensors: file shorter than 8 bytes"};
    uint64_t n = 0;
    for (int k = 7; k >= 0; --k) n = (n << 8) | len8[k];
    if (n > (1ull << 30)) throw Fail{FOPT_ERR_INVALID, "safetensors: header length implausible"};
    std::string text(n, '\0');
    if (n && fread(&text[0], 1, n, f) != n) throw Fail{FOPT_ERR_INVALID, "safetensors: header truncated"};
    fseek(f, 0, SEEK_END);
    st->file_size = (int64_t)ftell(f);
    st->data_start = 8 + (int64_t)n;
    parse_header(text, *st);
    for (auto& e : st->entries)
      if (st->data_start + e.end > st->file_size) throw Fail{FOPT_ERR_INVALID, "safetensors: " + e.name + " past the end"};
  } catch (const Fail& e) {
    fclose(f);
    delete st;
    g_noctx_err = e.msg;
    return e.code;
  } catch (const std::exception& e) {
    fclose(f);
    delete st;
    g_noctx_err = std::string("safetensors: ") + e.what();
    return FOPT_ERR_INVALID;
  }
  fclose(f);
  *out = st;
  return FOPT_OK;
}

fopt_status fopt_st_close(fopt_safetensors* st) {
  delete st;
  return FOPT_OK;
}

int32_t fopt_st_count(const fopt_safetensors* st) { return st ? (int32_t)st->entries.size() : 0; }

fopt_status fopt_st_info(const fopt_safetensors* st, int32_t i, const char** name, const char** dtype, int32_t* ndim,
                         int64_t* shape, int32_t max_dims, int64_t* bytes) {
  if (!st || i < 0 || i >= (int32_t)st->entries.size()) return FOPT_ERR_INVALID;
  const auto& e = st->entries[i];
  if (name) *name = e.name.c_str();
  if (dtype) *dtype = e.dtype.c_str();
  if (ndim) *ndim = (int32_t)e.shape.size();
  if (shape)
    for (int32_t k = 0; k < (int32_t)e.shape.size() && k < max_dims; ++k) shape[k] = e.shape[k];
  if (bytes) *bytes = e.end - e.begin;
  return FOPT_OK;
}

fopt_status fopt_st_find(const fopt_safetensors* st, const char* name, int32_t* index) {
  if (!st || !name || !index) return FOPT_ERR_INVALID;
  for (size_t k = 0; k < st->entries.size(); ++k)
    if (st->entries[k].name == name) {
      *index = (int32_t)k;
      return FOPT_OK;
    }
  g_noctx_err = std::string("safetensors: no tensor named ") + name;
  return FOPT_ERR_INVALID;
}

fopt_status fopt_st_read(fopt_ctx* ctx, const fopt_safetensors* st, int32_t i, void* dst, size_t bytes) {
  return guarded(ctx, [&] {
    require(st && dst && i >= 0 && i < (int32_t)st->entries.size(), "fopt_st_read: bad arguments");
    const auto& e = st->entries[i];
    require((int64_t)bytes == e.end - e.begin, "fopt_st_read: byte count differs from the tensor's");
    FILE* f = fopen(st->path.c_str(), "rb");
    require(f != nullptr, "fopt_st_read: cannot reopen the file");
    for (int k = 0; k < 2; ++k) {
      if (!ctx->pinned[k]) cuda_check(cudaHostAlloc(&ctx->pinned[k], kChunk, cudaHostAllocDefault), "pinned staging");
      if (!ctx->pinned_ev[k]) cuda_check(cudaEventCreateWithFlags(&ctx->pinned_ev[k], cudaEventDisableTiming), "event");
    }
    bool ok = fseek(f, (long)(st->data_start + e.begin), SEEK_SET) == 0;
    size_t done = 0;
    int k = 0;
    while (ok && done < bytes) {
      const size_t n = std::min(kChunk, bytes - done);
      cuda_check(cudaEventSynchronize(ctx->pinned_ev[k]), "staging reuse");  // its last copy has finished
      ok = fread(ctx->pinned[k], 1, n, f) == n;
      if (!ok) break;
      cuda_check(cudaMemcpyAsync((char*)dst + done, ctx->pinned[k], n, cudaMemcpyHostToDevice, ctx->stream), "h2d");
      cuda_check(cudaEventRecord(ctx->pinned_ev[k], ctx->stream), "event record");
      done += n;
      k ^= 1;
    }
    fclose(f);
    require(ok, "fopt_st_read: short read");
  });
}

fopt_status fopt_mapping_flat_shape(const fopt_mapping* m, int64_t* dims, int32_t max_dims, int32_t* n) {
  if (!m || !n) return FOPT_ERR_INVALID;
  std::vector<int64_t> out;
  flat_shape(*m->m.root, out);
  *n = (int32_t)out.size();
  if (dims)
    for (int32_t k = 0; k < (int32_t)out.size() && k < max_dims; ++k) dims[k] = out[k];
  return FOPT_OK;
}

}  // extern "C"
