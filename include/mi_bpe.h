/*
 * mi_bpe.h -- C ABI of the byte-level BPE tokenizer (host code, libmi_bpe.so).
 *
 * The entry points carry the names and argument meaning of the reference's
 * Rust tokenizer (src/rust_tokenizer/src/lib.rs), so its ctypes binding
 * (src/rust_tokenizer.py) loads this library unchanged.  Text is UTF-8; the
 * split pattern is the reference's GPT-4 pattern (lib.rs:8-9), with the
 * Unicode letter / number / white-space classes of
 * mamba_integer_b200/tokenizer/unicode_classes.h.
 */
#ifndef MI_BPE_H
#define MI_BPE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
namespace mi_bpe { struct Tokenizer; }
typedef mi_bpe::Tokenizer MiBpeTokenizer;
extern "C" {
#else
typedef struct MiBpeTokenizer MiBpeTokenizer;
#endif

/* New empty tokenizer (no merges: bytes encode as themselves).
 * Replaces: tokenizer_new, src/rust_tokenizer/src/lib.rs:15-21. */
MiBpeTokenizer* tokenizer_new(void);

/* Replaces: tokenizer_free, lib.rs:22-25. */
void tokenizer_free(MiBpeTokenizer* t);

/* Learn vocab_size - 256 merges from the UTF-8 lines of a text file: count
 * the byte sequences of every piece of every line, then repeatedly merge the
 * most frequent adjacent pair (ties: the smallest pair; the reference breaks
 * them in hash-map order).  vocab_size <= 256 learns nothing.  0 or -1 (file
 * not readable).
 * Replaces: tokenizer_train, lib.rs:26-71. */
int tokenizer_train(MiBpeTokenizer* t, const char* input_path, uint32_t vocab_size);

/* Token ids of a NUL-terminated UTF-8 text: its pieces under the split
 * pattern, each merged greedily (the leftmost occurrence of the pair with
 * the lowest merged id, until no pair has a merge).  Returns a malloc'd array
 * of *out_len ids (free with tokenizer_free_ids); NULL with *out_len = 0 for
 * an empty result or text that is not UTF-8 (the reference aborts on it).
 * Replaces: tokenizer_encode, lib.rs:73-98. */
uint32_t* tokenizer_encode(MiBpeTokenizer* t, const char* text, size_t* out_len);

/* Replaces: tokenizer_free_ids, lib.rs:99-102. */
void tokenizer_free_ids(uint32_t* ids, size_t len);

/* Write the merges as lines "a,b id" (sorted by id).  0 or -1.
 * Replaces: tokenizer_save, lib.rs:103-110 (which writes them in hash order). */
int tokenizer_save(MiBpeTokenizer* t, const char* path);

/* Add the merges of a file of lines "a,b id" (blank lines skipped).  0, or -1
 * for an unreadable file or a malformed line (the reference panics).
 * Replaces: tokenizer_load, lib.rs:111-123. */
int tokenizer_load(MiBpeTokenizer* t, const char* path);

/* The split alone: the byte offset where each piece of text ends, in order
 * (a piece starts where the previous one ends).  0; -1 if text is not UTF-8;
 * -2 if more than cap pieces (*n_out says how many).  No counterpart in the
 * reference (its pieces are internal to encode); used to test the split. */
int mi_bpe_pretokenize(const char* text, size_t* ends, size_t cap, size_t* n_out);

#ifdef __cplusplus
}
#endif
#endif /* MI_BPE_H */
