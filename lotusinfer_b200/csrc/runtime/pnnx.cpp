#include "pnnx.hpp"

#include <cctype>
#include <cstdio>
#include <memory>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace lotus {
namespace pnnx {

// ------------------------------------------------------------------ values
static bool looks_numeric(const std::string& v) {
  if (v.empty()) return false;
  if (v[0] == '-') return v.size() > 1 && (std::isdigit(static_cast<unsigned char>(v[1])) != 0);
  return std::isdigit(static_cast<unsigned char>(v[0])) != 0;
}
static bool looks_float(const std::string& v) {
  return v.find('.') != std::string::npos || v.find('e') != std::string::npos;
}

Parameter Parameter::Parse(const std::string& value) {
  Parameter p;
  if (value.find('%') != std::string::npos) {
    p.type = 4;
    p.s = value;
    return p;
  }
  if (value.empty() || value == "None" || value == "()" || value == "[]") return p;
  if (value == "True" || value == "False") {
    p.type = 1;
    p.b = value == "True";
    return p;
  }
  if (value[0] == '(' || value[0] == '[') {
    std::stringstream ss(value.substr(1, value.size() - 2));
    std::string e;
    while (std::getline(ss, e, ',')) {
      if (!looks_numeric(e)) {
        p.type = 7;
        p.as.push_back(e);
      } else if (looks_float(e)) {
        p.type = 6;
        p.af.push_back(std::stof(e));
      } else {
        p.type = 5;
        p.ai.push_back(std::stoi(e));
      }
    }
    return p;
  }
  if (!looks_numeric(value)) {
    p.type = 4;
    p.s = value;
  } else if (looks_float(value)) {
    p.type = 3;
    p.f = std::stof(value);
  } else {
    p.type = 2;
    p.i = std::stoi(value);
  }
  return p;
}

static void parse_shape(const std::string& v, std::vector<int>* shape, std::string* type) {
  const size_t close = v.find_last_of(')');
  if (v.empty() || v[0] != '(' || close == std::string::npos) throw std::runtime_error("bad shape '" + v + "'");
  *type = v.substr(close + 1);
  shape->clear();
  std::stringstream ss(v.substr(1, close - 1));
  std::string e;
  while (std::getline(ss, e, ',')) {
    if (e.empty()) continue;
    shape->push_back(e == "?" || e[0] == '%' ? -1 : std::stoi(e));
  }
}

// ------------------------------------------------------------------ zip
namespace {
uint16_t rd16(const unsigned char* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t rd32(const unsigned char* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
uint64_t rd64(const unsigned char* p) { return rd32(p) | (static_cast<uint64_t>(rd32(p + 4)) << 32); }

struct File {
  FILE* f;
  explicit File(const std::string& path) : f(std::fopen(path.c_str(), "rb")) {
    if (!f) throw std::runtime_error("cannot open " + path);
  }
  ~File() { std::fclose(f); }
  uint64_t size() {
    std::fseek(f, 0, SEEK_END);
    return static_cast<uint64_t>(ftello(f));
  }
  void read_at(uint64_t off, void* dst, size_t n) {
    if (fseeko(f, static_cast<off_t>(off), SEEK_SET) != 0 || std::fread(dst, 1, n, f) != n)
      throw std::runtime_error("short read in zip archive");
  }
};
}  // namespace

StoredZip::StoredZip(const std::string& path) : path_(path) {
  File file(path);
  const uint64_t fsize = file.size();
  if (fsize < 22) throw std::runtime_error(path + ": not a zip archive");
  // locate the end-of-central-directory record (last 22 + up to 64K comment bytes)
  const uint64_t tail = fsize < 65557 ? fsize : 65557;
  std::vector<unsigned char> buf(tail);
  file.read_at(fsize - tail, buf.data(), tail);
  int64_t eocd = -1;
  for (int64_t i = static_cast<int64_t>(tail) - 22; i >= 0; --i) {
    if (rd32(&buf[i]) == 0x06054b50u) {
      eocd = i;
      break;
    }
  }
  if (eocd < 0) throw std::runtime_error(path + ": end of central directory not found");
  uint64_t n_entries = rd16(&buf[eocd + 10]);
  uint64_t cd_size = rd32(&buf[eocd + 12]);
  uint64_t cd_off = rd32(&buf[eocd + 16]);
  if (cd_off == 0xFFFFFFFFu || n_entries == 0xFFFFu || cd_size == 0xFFFFFFFFu) {
    // zip64: locator sits right before the EOCD record
    if (eocd < 20 || rd32(&buf[eocd - 20]) != 0x07064b50u) throw std::runtime_error(path + ": zip64 locator missing");
    const uint64_t z64_off = rd64(&buf[eocd - 20 + 8]);
    unsigned char z[56];
    file.read_at(z64_off, z, sizeof(z));
    if (rd32(z) != 0x06064b50u) throw std::runtime_error(path + ": bad zip64 end record");
    n_entries = rd64(z + 32);
    cd_size = rd64(z + 40);
    cd_off = rd64(z + 48);
  }
  std::vector<unsigned char> cd(cd_size);
  file.read_at(cd_off, cd.data(), cd_size);
  size_t p = 0;
  for (uint64_t e = 0; e < n_entries; ++e) {
    if (p + 46 > cd.size() || rd32(&cd[p]) != 0x02014b50u) throw std::runtime_error(path + ": bad central directory");
    const uint16_t method = rd16(&cd[p + 10]);
    uint64_t csize = rd32(&cd[p + 20]);
    uint64_t usize = rd32(&cd[p + 24]);
    const uint16_t nlen = rd16(&cd[p + 28]), xlen = rd16(&cd[p + 30]), clen = rd16(&cd[p + 32]);
    uint64_t lho = rd32(&cd[p + 42]);
    const std::string name(reinterpret_cast<const char*>(&cd[p + 46]), nlen);
    // zip64 extra field: the 0xFFFFFFFF fields follow in order usize, csize, offset
    size_t x = p + 46 + nlen;
    const size_t xend = x + xlen;
    while (x + 4 <= xend) {
      const uint16_t id = rd16(&cd[x]), sz = rd16(&cd[x + 2]);
      if (id == 0x0001) {
        size_t q = x + 4;
        if (usize == 0xFFFFFFFFu) { usize = rd64(&cd[q]); q += 8; }
        if (csize == 0xFFFFFFFFu) { csize = rd64(&cd[q]); q += 8; }
        if (lho == 0xFFFFFFFFu) { lho = rd64(&cd[q]); q += 8; }
      }
      x += 4 + sz;
    }
    if (method != 0 || csize != usize) throw std::runtime_error(path + ": entry '" + name + "' is compressed");
    unsigned char lh[30];
    file.read_at(lho, lh, sizeof(lh));
    if (rd32(lh) != 0x04034b50u) throw std::runtime_error(path + ": bad local header");
    const uint64_t data_off = lho + 30 + rd16(lh + 26) + rd16(lh + 28);
    entries_[name] = Entry{data_off, usize};
    p += 46 + nlen + xlen + clen;
  }
}

uint64_t StoredZip::SizeOf(const std::string& name) const {
  auto it = entries_.find(name);
  return it == entries_.end() ? 0 : it->second.size;
}

std::vector<char> StoredZip::Read(const std::string& name) const {
  auto it = entries_.find(name);
  if (it == entries_.end()) throw std::runtime_error(path_ + ": no entry '" + name + "'");
  std::vector<char> out(it->second.size);
  File file(path_);
  if (!out.empty()) file.read_at(it->second.data_offset, out.data(), out.size());
  return out;
}

std::vector<std::string> StoredZip::Names() const {
  std::vector<std::string> n;
  for (auto& kv : entries_) n.push_back(kv.first);
  return n;
}

// ------------------------------------------------------------------ graph
static size_t elem_size(const std::string& t) {
  if (t == "f32" || t == "i32") return 4;
  if (t == "f16" || t == "bf16" || t == "i16") return 2;
  if (t == "f64" || t == "i64") return 8;
  if (t == "i8" || t == "u8" || t == "bool") return 1;
  return 0;
}

void Graph::Load(const std::string& param_path, const std::string& bin_path) {
  std::ifstream is(param_path);
  if (!is.good()) throw std::runtime_error("cannot open " + param_path);
  std::unique_ptr<StoredZip> zip;
  if (!bin_path.empty()) zip.reset(new StoredZip(bin_path));
  std::string line;
  std::getline(is, line);  // magic
  std::getline(is, line);
  int n_ops = 0, n_operands = 0;
  {
    std::istringstream ss(line);
    ss >> n_ops >> n_operands;
  }
  ops.clear();
  operands.clear();
  for (int k = 0; k < n_ops; ++k) {
    if (!std::getline(is, line)) throw std::runtime_error(param_path + ": truncated");
    std::istringstream ss(line);
    Operator op;
    int nin = 0, nout = 0;
    ss >> op.type >> op.name >> nin >> nout;
    for (int i = 0; i < nin; ++i) {
      std::string n;
      ss >> n;
      op.inputs.push_back(n);
      operands[n].name = n;
      operands[n].consumers.push_back(op.name);
    }
    for (int i = 0; i < nout; ++i) {
      std::string n;
      ss >> n;
      op.outputs.push_back(n);
      operands[n].name = n;
      operands[n].producer = op.name;
    }
    std::string item;
    while (ss >> item) {
      const size_t eq = item.find('=');
      if (eq == std::string::npos) continue;
      const std::string key = item.substr(0, eq), val = item.substr(eq + 1);
      if (key[0] == '@') {
        Attribute a;
        parse_shape(val, &a.shape, &a.type);
        const std::string entry = op.name + "." + key.substr(1);
        if (zip && zip->Has(entry)) {
          size_t expect = elem_size(a.type);
          for (int d : a.shape) expect *= static_cast<size_t>(d);
          if (zip->SizeOf(entry) != expect)
            throw std::runtime_error("attribute " + entry + ": size does not match its shape");
          a.data = zip->Read(entry);
        }
        op.attrs[key.substr(1)] = std::move(a);
      } else if (key[0] == '#') {
        OperandInfo& o = operands[key.substr(1)];
        o.name = key.substr(1);
        parse_shape(val, &o.shape, &o.type);
      } else if (key[0] == '$') {
        continue;
      } else {
        op.params[key] = Parameter::Parse(val);
      }
    }
    ops.push_back(std::move(op));
  }
}

}  // namespace pnnx
}  // namespace lotus
