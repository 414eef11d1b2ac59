// Unit tests of the host layer's JSON reader (flashmlx_b200/host/json.hpp), built and run
// by tests/test_host_cpp.py: objects, arrays, escapes (including surrogate pairs), numbers,
// literals, repeated keys, nesting limits and malformed documents.  Prints "ok" and exits
// 0 when every check holds; prints the failed check and exits 1 otherwise.
#include <cmath>
#include <cstdio>
#include <string>

#include "json.hpp"

using flashmoe::json::parse;
using flashmoe::json::Value;

static int failures = 0;

#define CHECK(cond)                                                     \
  do {                                                                  \
    if (!(cond)) {                                                      \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);     \
      ++failures;                                                       \
    }                                                                   \
  } while (0)

static bool throws(const std::string& doc) {
  try {
    parse(doc);
  } catch (const std::exception&) {
    return true;
  }
  return false;
}

int main() {
  // a safetensors-style header
  const Value h = parse(R"({"w": {"dtype": "U32", "shape": [2, 3], "data_offsets": [0, 24]},
                            "__metadata__": {"format": "mlx"}})");
  CHECK(h.is_object() && h.has("w") && h.has("__metadata__"));
  const Value* w = h.find("w");
  CHECK(w && w->string_or("dtype", "") == "U32");
  CHECK(w->find("shape")->arr.size() == 2 && w->find("shape")->arr[1].num == 3);
  CHECK(w->find("data_offsets")->arr[1].num == 24);

  // numbers: integers, negatives, exponents, large exact integers
  const Value n = parse(R"({"a": 4096, "b": -1e-6, "c": 1.5E3, "d": 9007199254740992, "e": 0})");
  CHECK(n.number_or("a", 0) == 4096);
  CHECK(std::fabs(n.number_or("b", 0) + 1e-6) < 1e-18);
  CHECK(n.number_or("c", 0) == 1500);
  CHECK(n.number_or("d", 0) == 9007199254740992.0);
  CHECK(n.number_or("missing", 7) == 7);

  // literals, null as absent, booleans read as numbers and back
  const Value l = parse(R"({"t": true, "f": false, "z": null, "one": 1})");
  CHECK(l.bool_or("t", false) && !l.bool_or("f", true));
  CHECK(l.number_or("z", 5) == 5 && l.bool_or("z", true));
  CHECK(l.bool_or("one", false) && l.number_or("t", 0) == 1);

  // escapes: quotes, backslash, control characters, \u with a surrogate pair
  const Value s = parse(R"({"s": "a\"b\\c\/d\n\t", "u": "\u00e9\u4E2D\ud83d\ude00"})");
  CHECK(s.string_or("s", "") == std::string("a\"b\\c/d\n\t"));
  CHECK(s.string_or("u", "") == std::string("\xc3\xa9\xe4\xb8\xad\xf0\x9f\x98\x80"));

  // a repeated key keeps the last value; whitespace everywhere
  const Value r = parse(" { \"k\" : 1 , \"k\" : 2 } ");
  CHECK(r.number_or("k", 0) == 2);

  // empty containers, nested arrays
  const Value e = parse(R"({"o": {}, "a": [], "n": [[1, [2]], {"x": [3]}]})");
  CHECK(e.find("o")->is_object() && e.find("o")->obj.empty() && e.find("a")->arr.empty());
  CHECK(e.find("n")->arr[0].arr[1].arr[0].num == 2);

  // type errors are reported, not coerced
  bool threw = false;
  try {
    parse(R"({"a": "x"})").number_or("a", 0);
  } catch (const std::exception&) {
    threw = true;
  }
  CHECK(threw);

  // malformed documents
  CHECK(throws(""));
  CHECK(throws("{"));
  CHECK(throws(R"({"a": 1,})"));
  CHECK(throws(R"({"a" 1})"));
  CHECK(throws(R"({"a": tru})"));
  CHECK(throws(R"({"a": "unterminated})"));
  CHECK(throws(R"({"a": "\x"})"));
  CHECK(throws(R"({"a": "\u12"})"));
  CHECK(throws(R"({"a": 1} trailing)"));
  CHECK(throws(R"({"a": --1})"));
  CHECK(throws(std::string(70, '[') + std::string(70, ']')));  // nesting past 64 levels

  if (failures) return 1;
  std::printf("ok\n");
  return 0;
}
