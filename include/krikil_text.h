/*
 * krikil_text.h -- C ABI of the text front end that turns a user prompt into
 * token ids and generated ids back into text: the tokenizer
 * (src/tokenizer.rs, a byte-level BPE read from tokenizer.json) and the chat
 * template (src/template.rs).  Host code in the same library as
 * krikil_cuda.h; none of these calls touches a GPU.
 *
 * Same conventions as krikil_cuda.h: every function returns a krk_status and
 * sets krk_last_error() on failure; host buffers belong to the caller.
 * Output buffers follow one rule: *len_out (or *n_out) always receives the
 * full size of the result; when the buffer pointer is NULL nothing is
 * written (a size query); when it is too small the call fails with
 * KRK_INVALID.  Strings are UTF-8; output strings get a terminating NUL when
 * the buffer has room for it (not counted in *len_out).
 */
#ifndef KRIKIL_TEXT_H
#define KRIKIL_TEXT_H

#include "krikil_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct krk_tokenizer krk_tokenizer;

/* PebbleTokenizer::from_file (src/tokenizer.rs:14-23).  KRK_IO with
 * "Failed to load tokenizer from <path>: <why>" if the file is missing,
 * unreadable or not a supported tokenizer.json. */
KRK_API int krk_tokenizer_load(const char* path, krk_tokenizer** out);
KRK_API int krk_tokenizer_free(krk_tokenizer* tok);

/* PebbleTokenizer::encode (src/tokenizer.rs:25-32): `len` bytes of UTF-8
 * text -> token ids (no special tokens added).  At most `len` ids result.
 * KRK_INVALID with "Failed to encode text: ..." for invalid UTF-8. */
KRK_API int krk_tokenizer_encode(const krk_tokenizer* tok, const char* text, size_t len, uint32_t* ids,
                                 size_t cap, size_t* n_out);

/* PebbleTokenizer::decode (skip_special = 1, src/tokenizer.rs:34-38) and
 * decode_token (skip_special = 0, one id, src/tokenizer.rs:40-44): ids ->
 * UTF-8 text; ids outside the vocabulary are skipped, bytes that do not form
 * UTF-8 become U+FFFD. */
KRK_API int krk_tokenizer_decode(const krk_tokenizer* tok, const uint32_t* ids, size_t n, int skip_special,
                                 char* out, size_t cap, size_t* len_out);

/* Tokenizer::token_to_id: *id = the token's id, or -1 if it has none. */
KRK_API int krk_tokenizer_token_to_id(const krk_tokenizer* tok, const char* token, int64_t* id);
/* PebbleTokenizer::eos_token_id (src/tokenizer.rs:46-48): the id of
 * "<|eos|>", or 0 (DEFAULT_EOS_TOKEN_ID) if the vocabulary has none. */
KRK_API int krk_tokenizer_eos_token_id(const krk_tokenizer* tok, uint32_t* id);
/* PebbleTokenizer::vocab_size (src/tokenizer.rs:50-52), added tokens included. */
KRK_API int krk_tokenizer_vocab_size(const krk_tokenizer* tok, size_t* n);

/* PebbleTokenizer::resolve_path (src/tokenizer.rs:54-79): explicit_path if
 * given (KRK_IO if it does not exist), else tokenizer.json beside the model
 * file, else ./tokenizer.json, else KRK_IO with the reference's message. */
KRK_API int krk_tokenizer_resolve_path(const char* model_path, const char* explicit_path, char* out, size_t cap,
                                       size_t* len_out);

/* ChatTemplateEngine::render (src/template.rs:59-73) of `source` (NULL: the
 * built-in DEFAULT_CHAT_TEMPLATE, src/template.rs:7) over n messages
 * (roles[i], contents[i]) with add_generation_prompt.  KRK_INVALID with
 * "Failed to parse Jinja chat template: ..." or "Failed to render Jinja chat
 * template: ..." on errors. */
KRK_API int krk_chat_template_render(const char* source, const char* const* roles, const char* const* contents,
                                     size_t n, int add_generation_prompt, char* out, size_t cap, size_t* len_out);

/* The built-in template text (static storage). */
KRK_API const char* krk_default_chat_template(void);

#ifdef __cplusplus
}
#endif

#endif /* KRIKIL_TEXT_H */
