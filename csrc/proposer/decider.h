// Decision-endpoint helpers (CPU, no GPU state): prompt construction for a
// classifier that reads one logit per answer code, and the reduction of those
// logits to answers.  Behaviour of the reference's decider helpers
// (src/pplx_decider.rs:100-420, bound as decider_prepare / decider_answer at
// src/lib.rs:431-443): JSON in, JSON out, question and option order preserved
// (option i is read out from logit row entry i), prompts rendered exactly like
// Python's json.dumps(..., ensure_ascii=False).  Two prompt profiles: "pplx"
// (text only) and "d3" (any JSON descriptions, image / video placeholders).
#pragma once
#include <string>

namespace sh {

// request JSON + answer codes JSON list + profile -> {"rows": [{"messages", "option_count"}], "identifiers"}.
// Throws std::invalid_argument on a malformed request.
std::string decider_prepare(const std::string& request_json, const std::string& codes_json,
                            const std::string& profile);
// request JSON + logits JSON ([questions][options..]) + temperature + profile ->
// {"model", "answers": {id: {...}}, "usage"}.  Throws std::invalid_argument.
std::string decider_answer(const std::string& request_json, const std::string& logits_json, double temperature,
                           const std::string& profile);

}  // namespace sh
