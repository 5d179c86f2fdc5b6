// OpenAI tool calling for the chat route: the tools preamble rendered into the prompt and the
// extraction of tool calls from a completion.
//
// Preamble (Hermes / Qwen style): the function signatures inside <tools></tools> and the
// instruction to answer with {"name": ..., "arguments": {...}} inside <tool_call></tool_call>.
// Extraction: every tagged <tool_call> block (explicit intent, lenient: a block without its
// closing tag runs to the end of the text); without tags, the first JSON object (or array of
// objects) in the text whose "name" is one of the request's declared tools, so a plain answer
// that merely contains a JSON object is not read as a call. Arguments are returned as a JSON-
// encoded string, as the OpenAI schema carries them.
//
// Parity: crates/hawking-serve/src/tool_calls.rs:43-123 (render_tools_preamble, tool_names,
// extract_tool_calls).
#pragma once
#include <string>
#include <vector>

#include "json.h"

namespace hk {

struct ToolCall {
  std::string id, name, arguments;
};

std::string render_tools_preamble(const Json& tools);
std::vector<std::string> tool_names(const Json& tools);
std::vector<ToolCall> extract_tool_calls(const std::string& completion, const std::vector<std::string>& known_tools);

}  // namespace hk
