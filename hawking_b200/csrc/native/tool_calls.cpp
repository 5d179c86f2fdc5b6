#include "tool_calls.h"

#include <utility>

namespace hk {

std::string render_tools_preamble(const Json& tools) {
  if (!tools.is_array() || tools.size() == 0) return std::string();
  std::string s =
      "# Tools\n\nYou may call one or more functions to assist with the user query.\n\n"
      "You are provided with function signatures within <tools></tools> XML tags:\n<tools>\n";
  for (const auto& t : tools.items()) {
    const Json& f = t.has("function") ? t["function"] : t;  // OpenAI envelope or bare function
    s += f.dump();
    s += '\n';
  }
  s +=
      "</tools>\n\nFor each function call, return a json object with the function name and arguments within "
      "<tool_call></tool_call> XML tags:\n<tool_call>\n{\"name\": <function-name>, \"arguments\": "
      "<args-json-object>}\n</tool_call>\n";
  return s;
}

std::vector<std::string> tool_names(const Json& tools) {
  std::vector<std::string> out;
  if (!tools.is_array()) return out;
  for (const auto& t : tools.items()) {
    const Json& f = t.has("function") ? t["function"] : t;
    if (f.is_object() && f["name"].is_string()) out.push_back(f["name"].as_string());
  }
  return out;
}

namespace {

// Balanced {...} / [...] spans outside JSON strings, in document order (outermost only).
std::vector<std::string> json_spans(const std::string& s) {
  std::vector<std::string> out;
  size_t i = 0;
  while (i < s.size()) {
    if (s[i] != '{' && s[i] != '[') {
      ++i;
      continue;
    }
    int depth = 0;
    bool in_str = false, esc = false;
    size_t j = i;
    for (; j < s.size(); ++j) {
      const char c = s[j];
      if (in_str) {
        if (esc) esc = false;
        else if (c == '\\') esc = true;
        else if (c == '"') in_str = false;
        continue;
      }
      if (c == '"') in_str = true;
      else if (c == '{' || c == '[') ++depth;
      else if (c == '}' || c == ']') {
        if (--depth == 0) break;
      }
    }
    if (j < s.size()) {
      out.push_back(s.substr(i, j - i + 1));
      i = j + 1;
    } else {
      break;  // unbalanced tail
    }
  }
  return out;
}

bool try_parse(const std::string& text, Json& out) {
  try {
    out = Json::parse(text);
    return true;
  } catch (...) {
    return false;
  }
}

// (name, arguments) pairs of a parsed value: one call object or an array of them.
void calls_from_value(const Json& v, std::vector<std::pair<std::string, Json>>& out) {
  if (v.is_array()) {
    for (const auto& e : v.items()) calls_from_value(e, out);
    return;
  }
  if (!v.is_object() || !v["name"].is_string()) return;
  Json args = v.has("arguments") ? v["arguments"] : (v.has("parameters") ? v["parameters"] : Json::object());
  if (args.is_string()) {  // already JSON-encoded: keep the object when it parses
    Json parsed;
    if (try_parse(args.as_string(), parsed)) args = parsed;
  }
  out.emplace_back(v["name"].as_string(), args);
}

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (s[a] == ' ' || s[a] == '\n' || s[a] == '\r' || s[a] == '\t')) ++a;
  while (b > a && (s[b - 1] == ' ' || s[b - 1] == '\n' || s[b - 1] == '\r' || s[b - 1] == '\t')) --b;
  return s.substr(a, b - a);
}

}  // namespace

std::vector<ToolCall> extract_tool_calls(const std::string& completion, const std::vector<std::string>& known) {
  static const std::string open = "<tool_call>", close = "</tool_call>";
  std::vector<std::pair<std::string, Json>> raw;
  size_t at = completion.find(open);
  bool tagged = false;
  while (at != std::string::npos) {
    tagged = true;
    const size_t body = at + open.size();
    const size_t end = completion.find(close, body);
    const std::string inner = trim(completion.substr(body, end == std::string::npos ? std::string::npos : end - body));
    Json v;
    if (try_parse(inner, v)) calls_from_value(v, raw);
    else
      for (const auto& span : json_spans(inner))
        if (try_parse(span, v)) {
          calls_from_value(v, raw);
          break;
        }
    if (end == std::string::npos) break;
    at = completion.find(open, end + close.size());
  }
  if (!tagged) {
    for (const auto& span : json_spans(completion)) {
      Json v;
      if (!try_parse(span, v)) continue;
      std::vector<std::pair<std::string, Json>> found;
      calls_from_value(v, found);
      std::vector<std::pair<std::string, Json>> keep;
      for (auto& c : found)
        for (const auto& k : known)
          if (c.first == k) {
            keep.push_back(c);
            break;
          }
      if (!keep.empty()) {
        raw = std::move(keep);
        break;
      }
    }
  }
  std::vector<ToolCall> out;
  for (size_t i = 0; i < raw.size(); ++i) out.push_back({"call_" + std::to_string(i), raw[i].first, raw[i].second.dump()});
  return out;
}

}  // namespace hk
