// PNNX model reader: the `.pnnx.param` text graph plus the stored-zip
// `.pnnx.bin` weight archive, the on-disk format the reference loads through
// its vendored ncnn/PNNX code (source/pnnx/ir.cpp:700-806 for the text,
// source/pnnx/storezip.cpp:143-317 for the archive).
//
// Format facts kept identical: line 1 magic, line 2 "op_count operand_count",
// then one operator per line "type name n_in n_out <in names> <out names>
// key=value..." where '@key=(shape)type' names an attribute stored in the
// archive as entry "<op name>.<key>", '#name=(shape)type' gives an operand
// shape and '$key=name' an input key; parameter values parse like
// Parameter::parse_from_string (source/pnnx/ir.cpp:327-406).
// The archive reader here walks the zip central directory (with zip64
// extensions) rather than scanning local headers.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace lotus {
namespace pnnx {

struct Parameter {
  // 0 none, 1 bool, 2 int, 3 float, 4 string, 5 int list, 6 float list, 7 string list
  int type = 0;
  bool b = false;
  int i = 0;
  float f = 0.f;
  std::string s;
  std::vector<int> ai;
  std::vector<float> af;
  std::vector<std::string> as;
  static Parameter Parse(const std::string& value);
};

struct Attribute {
  std::string type;            // "f32", ...
  std::vector<int> shape;
  std::vector<char> data;      // raw bytes from the archive (empty if absent)
};

struct OperandInfo {
  std::string name;
  std::string type;            // "f32", ...
  std::vector<int> shape;
  std::string producer;
  std::vector<std::string> consumers;
};

struct Operator {
  std::string type;
  std::string name;
  std::vector<std::string> inputs;
  std::vector<std::string> outputs;
  std::map<std::string, Parameter> params;
  std::map<std::string, Attribute> attrs;
};

// Minimal reader of a zip archive whose entries are stored (not deflated).
class StoredZip {
 public:
  // Throws std::runtime_error on malformed or compressed archives.
  explicit StoredZip(const std::string& path);
  bool Has(const std::string& name) const { return entries_.count(name) != 0; }
  uint64_t SizeOf(const std::string& name) const;
  std::vector<char> Read(const std::string& name) const;
  std::vector<std::string> Names() const;

 private:
  struct Entry {
    uint64_t data_offset;
    uint64_t size;
  };
  std::string path_;
  std::map<std::string, Entry> entries_;
};

struct Graph {
  std::vector<Operator> ops;                      // in file order
  std::map<std::string, OperandInfo> operands;
  // Parses param_path; attribute data are read from bin_path ("" = none).
  void Load(const std::string& param_path, const std::string& bin_path);
};

}  // namespace pnnx
}  // namespace lotus
