// chat_template.h -- renders chat templates, the prompt front end of the CLI
// (src/template.rs:34-79 renders them with minijinja 2.x).
//
// The template language is the Jinja subset chat templates use:
//   {{ expr }}, {% if %}/{% elif %}/{% else %}/{% endif %},
//   {% for x in expr %} (also "for a, b in", an "else" branch and the loop
//   variable: index, index0, revindex, revindex0, first, last, length),
//   {% set name = expr %}, {# comments #}, "-" whitespace control;
// expressions with string / number / true / false / none literals and lists,
// variables, .attr and [key] access and [a:b] slices, not / and / or,
// == != < > <= >= in / not in, ~ + - * / // %, "a if c else b",
// "is [not] <test>" (defined, undefined, none, string, number, integer,
// float, boolean, true, false, mapping, sequence, iterable, odd, even), the
// filters length/count, trim, upper, lower, capitalize, default/d, first,
// last, string, int, join, list, reverse, and the functions range() and
// raise_exception().  As in minijinja's defaults: no auto-escaping, undefined
// values print as "" and are false, a single trailing newline of the
// template is dropped.  Host code only.
#pragma once

#include <string>
#include <vector>

namespace krk {

struct ChatMessage {
    std::string role;
    std::string content;
};

// src/template.rs:7
extern const char* const DEFAULT_CHAT_TEMPLATE;

// ChatTemplateEngine::render (src/template.rs:59-73): the template with
// `messages` and `add_generation_prompt` in its context.  On failure returns
// false with err = "Failed to parse Jinja chat template: ..." or
// "Failed to render Jinja chat template: ...".
bool render_chat_template(const std::string& source, const std::vector<ChatMessage>& messages,
                          bool add_generation_prompt, std::string& out, std::string& err);

}  // namespace krk
