// tokenizer.cu — upstream's byte-level BPE tokenizer, on the host.
//
// The tokenizer is not on the GPU path (upstream runs it once per prompt and
// once per generated token for text output); it is here so that upstream's
// callers (examples/generate_example.c, q_generate's callers) link against
// this library alone.  Semantics of upstream src/tokenizer/bpe.c:
//   * file: 8 little-endian u32 (magic 'QTKR', version 1, vocab size, merge
//     count, BOS, EOS, PAD, reserved), then per token a u8 length (> 0) and
//     its bytes, then per merge three u32 (first, second, merged) — bpe.c:279-487;
//   * encode: every byte of the text is a token id (its value; PAD when the
//     value is not below the vocabulary size), then the merge rules are
//     applied in priority order, each scanning the live tokens left to
//     right, and the whole pass repeats until nothing changes; optional BOS
//     in front and EOS at the end — bpe.c:492-799;
//   * the merged id of a pair comes from a table keyed (first << 16) | second
//     in which a later rule with the same key replaces an earlier one
//     (bpe.c:106-215; for vocabularies past 65536 ids distinct pairs can share
//     a key, and upstream then takes the later rule's id — kept, so encodes
//     are identical);
//   * decode: concatenation of the tokens' strings, BOS/EOS/PAD and ids past
//     the vocabulary skipped — bpe.c:803-857.
// Error codes follow upstream's.
#include <cstdio>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "qorus.h"

namespace {

constexpr uint32_t kTokMagic = 0x51544B52u;  // 'QTKR'
constexpr uint32_t kTokVersion = 1;
constexpr size_t kMaxTextBytes = 1024 * 1024;
constexpr uint32_t kDeleted = 0xFFFFFFFFu;

struct MergeTable {
    std::unordered_map<uint64_t, uint32_t> merged;  // (first << 16) | second -> merged id (last rule wins)
};

bool read_u32(FILE* f, uint32_t* v) {
    uint8_t b[4];
    if (fread(b, 1, 4, f) != 4) return false;
    *v = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    return true;
}

void release(q_tokenizer* tok) {
    if (tok->vocab) {
        for (uint32_t i = 0; i < tok->vocab_size; ++i) free(tok->vocab[i]);
        free((void*)tok->vocab);
    }
    free(tok->merges);
    delete reinterpret_cast<MergeTable*>(tok->merge_hash_table);
    memset(tok, 0, sizeof *tok);
}

}  // namespace

extern "C" {

q_error_code q_tokenizer_load(q_tokenizer* tok, const char* path) {
    if (!tok || !path) return Q_ERR_INVALID_ARG;
    memset(tok, 0, sizeof *tok);
    FILE* f = fopen(path, "rb");
    if (!f) return Q_ERR_FILE_OPEN;
    // Header words are read and checked in order, so a short file with a bad
    // magic reports the magic, as upstream's loader does.
    uint32_t h[8];
    q_error_code rc = Q_OK;
    for (int i = 0; i < 8 && rc == Q_OK; ++i) {
        if (!read_u32(f, &h[i])) rc = Q_ERR_FILE_OPEN;
        else if (i == 0 && h[0] != kTokMagic) rc = Q_ERR_INVALID_MAGIC;
        else if (i == 1 && h[1] != kTokVersion) rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && (h[2] == 0 || h[2] > 1000000 || h[3] > 1000000)) rc = Q_ERR_INVALID_SIZE;
    if (rc != Q_OK) {
        fclose(f);
        return rc;
    }
    tok->vocab_size = h[2];
    tok->num_merges = h[3];
    tok->bos_token_id = h[4];
    tok->eos_token_id = h[5];
    tok->pad_token_id = h[6];
    tok->vocab = (char**)calloc(tok->vocab_size, sizeof(char*));
    if (!tok->vocab) {
        fclose(f);
        memset(tok, 0, sizeof *tok);
        return Q_ERR_ALLOC_FAILED;
    }
    for (uint32_t i = 0; i < tok->vocab_size && rc == Q_OK; ++i) {
        uint8_t len = 0;
        if (fread(&len, 1, 1, f) != 1) rc = Q_ERR_FILE_OPEN;
        else if (len == 0) rc = Q_ERR_INVALID_SIZE;
        else if (!(tok->vocab[i] = (char*)malloc((size_t)len + 1))) rc = Q_ERR_ALLOC_FAILED;
        else if (fread(tok->vocab[i], 1, len, f) != len) rc = Q_ERR_FILE_OPEN;
        else tok->vocab[i][len] = '\0';
    }
    if (rc == Q_OK && tok->num_merges) {
        tok->merges = (q_bpe_merge*)calloc(tok->num_merges, sizeof(q_bpe_merge));
        if (!tok->merges) rc = Q_ERR_ALLOC_FAILED;
        for (uint32_t i = 0; i < tok->num_merges && rc == Q_OK; ++i) {
            q_bpe_merge& m = tok->merges[i];
            if (!read_u32(f, &m.token_id1) || !read_u32(f, &m.token_id2) || !read_u32(f, &m.merged_id))
                rc = Q_ERR_FILE_OPEN;
            else if (m.token_id1 >= tok->vocab_size || m.token_id2 >= tok->vocab_size ||
                     m.merged_id >= tok->vocab_size)
                rc = Q_ERR_INVALID_ARG;
        }
        if (rc == Q_OK) {
            MergeTable* t = new MergeTable;
            t->merged.reserve((size_t)tok->num_merges * 2);
            for (uint32_t i = 0; i < tok->num_merges; ++i)
                t->merged[((uint64_t)tok->merges[i].token_id1 << 16) | tok->merges[i].token_id2] =
                    tok->merges[i].merged_id;
            tok->merge_hash_table = reinterpret_cast<struct bpe_hash_table*>(t);
        }
    }
    fclose(f);
    if (rc != Q_OK) {
        release(tok);
        return rc;
    }
    tok->initialized = true;
    return Q_OK;
}

q_error_code q_tokenizer_encode(q_tokenizer* tok, const char* text, uint32_t* tokens_out,
                                uint32_t* num_tokens_out, uint32_t max_tokens, bool add_bos, bool add_eos) {
    if (!tok || !text || !tokens_out || !num_tokens_out || !tok->initialized) return Q_ERR_INVALID_ARG;
    if (max_tokens == 0) return Q_ERR_INVALID_SIZE;
    const size_t n_text = strlen(text);
    if (n_text == 0) {
        const size_t need = (add_bos ? 1 : 0) + (add_eos ? 1 : 0);
        *num_tokens_out = 0;
        if (need > max_tokens) return Q_ERR_ARENA_OOM;
        uint32_t n = 0;
        if (add_bos) tokens_out[n++] = tok->bos_token_id;
        if (add_eos) tokens_out[n++] = tok->eos_token_id;
        *num_tokens_out = n;
        return Q_OK;
    }
    if (n_text > kMaxTextBytes) return Q_ERR_ARENA_OOM;
    const size_t cap = std::max(n_text, (size_t)max_tokens);
    std::vector<uint32_t> ids(cap);
    for (size_t i = 0; i < n_text; ++i) {
        const uint8_t b = (uint8_t)text[i];
        ids[i] = b < tok->vocab_size ? b : tok->pad_token_id;
    }
    size_t n = n_text;
    const MergeTable* table = reinterpret_cast<const MergeTable*>(tok->merge_hash_table);
    if (tok->num_merges && n >= 2) {
        size_t deleted = 0;
        const size_t compact_at = n / 2;
        for (bool changed = true; changed;) {
            changed = false;
            for (uint32_t r = 0; r < tok->num_merges; ++r) {
                const uint32_t a = tok->merges[r].token_id1, b = tok->merges[r].token_id2;
                uint32_t merged = tok->merges[r].merged_id;
                if (table) {
                    auto it = table->merged.find(((uint64_t)a << 16) | b);
                    if (it != table->merged.end()) merged = it->second;
                }
                for (size_t j = 0; j < n; ++j) {
                    if (ids[j] == kDeleted) continue;
                    size_t nx = j + 1;
                    while (nx < n && ids[nx] == kDeleted) ++nx;
                    if (nx >= n) break;
                    if (ids[j] == a && ids[nx] == b) {
                        ids[j] = merged;
                        ids[nx] = kDeleted;
                        ++deleted;
                        changed = true;
                    }
                }
            }
            if (deleted > compact_at) {
                size_t w = 0;
                for (size_t i = 0; i < n; ++i)
                    if (ids[i] != kDeleted) ids[w++] = ids[i];
                n = w;
                deleted = 0;
            }
        }
        size_t w = 0;
        for (size_t i = 0; i < n; ++i)
            if (ids[i] != kDeleted) ids[w++] = ids[i];
        n = w;
    }
    const size_t need = n + (add_bos ? 1 : 0) + (add_eos ? 1 : 0);
    if (need > cap || need > max_tokens) return Q_ERR_ARENA_OOM;
    size_t o = 0;
    if (add_bos) tokens_out[o++] = tok->bos_token_id;
    memcpy(tokens_out + o, ids.data(), n * 4);
    o += n;
    if (add_eos) tokens_out[o++] = tok->eos_token_id;
    *num_tokens_out = (uint32_t)o;
    return Q_OK;
}

q_error_code q_tokenizer_decode(q_tokenizer* tok, const uint32_t* tokens, uint32_t num_tokens, char* text_out,
                                size_t text_buf_size) {
    if (!tok || !tokens || !text_out || !tok->initialized) return Q_ERR_INVALID_ARG;
    if (text_buf_size == 0) return Q_ERR_INVALID_SIZE;
    size_t pos = 0;
    for (uint32_t i = 0; i < num_tokens; ++i) {
        const uint32_t id = tokens[i];
        if (id == tok->bos_token_id || id == tok->eos_token_id || id == tok->pad_token_id) continue;
        if (id >= tok->vocab_size || !tok->vocab[id]) continue;
        const size_t len = strlen(tok->vocab[id]);
        if (pos + len >= text_buf_size - 1) {
            text_out[pos] = '\0';
            return Q_ERR_ARENA_OOM;
        }
        memcpy(text_out + pos, tok->vocab[id], len);
        pos += len;
    }
    text_out[pos] = '\0';
    return Q_OK;
}

void q_tokenizer_free(q_tokenizer* tok) {
    if (!tok) return;
    release(tok);
}

}  // extern "C"
