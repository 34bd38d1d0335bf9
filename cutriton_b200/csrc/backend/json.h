#pragma once

// Minimal JSON reader for Kernel Pack manifests. Strict: rejects trailing
// data, duplicate keys and unsupported escapes; numbers are doubles. Errors
// are thrown as std::runtime_error and converted to Status by the caller.

#include <cctype>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace cutriton {
namespace json {

struct Value {
  enum class Type { kNull, kBool, kNumber, kString, kArray, kObject };
  Type type{Type::kNull};
  bool boolean{false};
  double number{0.0};
  std::string text;
  std::vector<Value> items;
  std::map<std::string, Value> members;

  bool is_object() const { return type == Type::kObject; }
  const Value& at(const std::string& key) const {
    if (type != Type::kObject) throw std::runtime_error("expected an object around field " + key);
    const auto it = members.find(key);
    if (it == members.end()) throw std::runtime_error("missing field: " + key);
    return it->second;
  }
  const Value* find(const std::string& key) const {
    if (type != Type::kObject) return nullptr;
    const auto it = members.find(key);
    return it == members.end() ? nullptr : &it->second;
  }
  const std::string& str() const {
    if (type != Type::kString) throw std::runtime_error("expected a string");
    return text;
  }
  double num() const {
    if (type != Type::kNumber) throw std::runtime_error("expected a number");
    return number;
  }
  bool flag() const {
    if (type != Type::kBool) throw std::runtime_error("expected a boolean");
    return boolean;
  }
  const std::vector<Value>& list() const {
    if (type != Type::kArray) throw std::runtime_error("expected an array");
    return items;
  }
  const std::map<std::string, Value>& object() const {
    if (type != Type::kObject) throw std::runtime_error("expected an object");
    return members;
  }
};

class Reader {
 public:
  explicit Reader(const std::string& text) : text_(text) {}

  Value Document() {
    Value value = Parse(0);
    Skip();
    if (pos_ != text_.size()) throw std::runtime_error("trailing data after JSON document");
    return value;
  }

 private:
  void Skip() {
    while (pos_ < text_.size() && std::isspace(static_cast<unsigned char>(text_[pos_]))) ++pos_;
  }
  char Peek() {
    Skip();
    if (pos_ >= text_.size()) throw std::runtime_error("unexpected end of JSON");
    return text_[pos_];
  }
  void Expect(char c) {
    if (Peek() != c) throw std::runtime_error(std::string("expected '") + c + "'");
    ++pos_;
  }
  bool Literal(const char* word) {
    const std::string w(word);
    if (text_.compare(pos_, w.size(), w) == 0) {
      pos_ += w.size();
      return true;
    }
    return false;
  }

  Value Parse(int depth) {
    if (depth > 64) throw std::runtime_error("JSON nesting is too deep");
    Value v;
    const char c = Peek();
    if (c == '{') {
      v.type = Value::Type::kObject;
      ++pos_;
      if (Peek() == '}') { ++pos_; return v; }
      while (true) {
        if (Peek() != '"') throw std::runtime_error("expected an object key");
        std::string key = String();
        Expect(':');
        Value member = Parse(depth + 1);
        if (!v.members.emplace(std::move(key), std::move(member)).second) {
          throw std::runtime_error("duplicate object key");
        }
        if (Peek() == ',') { ++pos_; continue; }
        Expect('}');
        return v;
      }
    }
    if (c == '[') {
      v.type = Value::Type::kArray;
      ++pos_;
      if (Peek() == ']') { ++pos_; return v; }
      while (true) {
        v.items.push_back(Parse(depth + 1));
        if (Peek() == ',') { ++pos_; continue; }
        Expect(']');
        return v;
      }
    }
    if (c == '"') {
      v.type = Value::Type::kString;
      v.text = String();
      return v;
    }
    if (c == '-' || std::isdigit(static_cast<unsigned char>(c))) {
      v.type = Value::Type::kNumber;
      v.number = Number();
      return v;
    }
    if (Literal("true")) { v.type = Value::Type::kBool; v.boolean = true; return v; }
    if (Literal("false")) { v.type = Value::Type::kBool; v.boolean = false; return v; }
    if (Literal("null")) return v;
    throw std::runtime_error("invalid JSON value");
  }

  std::string String() {
    Expect('"');
    std::string out;
    while (true) {
      if (pos_ >= text_.size()) throw std::runtime_error("unterminated JSON string");
      const char c = text_[pos_++];
      if (c == '"') return out;
      if (c != '\\') { out.push_back(c); continue; }
      if (pos_ >= text_.size()) throw std::runtime_error("unterminated JSON escape");
      const char e = text_[pos_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        default: throw std::runtime_error("unsupported JSON escape");
      }
    }
  }

  double Number() {
    const std::size_t begin = pos_;
    if (text_[pos_] == '-') ++pos_;
    auto digits = [&]() {
      while (pos_ < text_.size() && std::isdigit(static_cast<unsigned char>(text_[pos_]))) ++pos_;
    };
    digits();
    if (pos_ < text_.size() && text_[pos_] == '.') { ++pos_; digits(); }
    if (pos_ < text_.size() && (text_[pos_] == 'e' || text_[pos_] == 'E')) {
      ++pos_;
      if (pos_ < text_.size() && (text_[pos_] == '+' || text_[pos_] == '-')) ++pos_;
      digits();
    }
    const std::string token = text_.substr(begin, pos_ - begin);
    char* end = nullptr;
    const double value = std::strtod(token.c_str(), &end);
    if (end == token.c_str() || *end != '\0') throw std::runtime_error("invalid JSON number");
    return value;
  }

  const std::string& text_;
  std::size_t pos_{0};
};

inline Value Parse(const std::string& text) { return Reader(text).Document(); }

}  // namespace json
}  // namespace cutriton
