/* The few declarations of the PCRE2 8-bit API (public documentation:
 * pcre2api(3)) that the reference's tokenizer uses
 * (src/models/qwen3/tokenizer.cpp:140-226), so that its unmodified source
 * compiles against the system's PCRE2 runtime (libpcre2-8.so.0, whose
 * development headers are not installed). Oracle builds only. */
#ifndef ORACLE_PCRE2_DECL_H
#define ORACLE_PCRE2_DECL_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint8_t PCRE2_UCHAR8;
typedef const PCRE2_UCHAR8* PCRE2_SPTR8;
typedef size_t PCRE2_SIZE;
typedef struct pcre2_real_code_8 pcre2_code_8;
typedef struct pcre2_real_match_data_8 pcre2_match_data_8;
typedef struct pcre2_real_general_context_8 pcre2_general_context_8;
typedef struct pcre2_real_compile_context_8 pcre2_compile_context_8;
typedef struct pcre2_real_match_context_8 pcre2_match_context_8;

#define PCRE2_UCP 0x00020000u
#define PCRE2_UTF 0x00080000u

pcre2_code_8* pcre2_compile_8(PCRE2_SPTR8 pattern, PCRE2_SIZE length, uint32_t options, int* errorcode,
                              PCRE2_SIZE* erroroffset, pcre2_compile_context_8* ccontext);
void pcre2_code_free_8(pcre2_code_8* code);
pcre2_match_data_8* pcre2_match_data_create_from_pattern_8(const pcre2_code_8* code, pcre2_general_context_8* gcontext);
void pcre2_match_data_free_8(pcre2_match_data_8* match_data);
int pcre2_match_8(const pcre2_code_8* code, PCRE2_SPTR8 subject, PCRE2_SIZE length, PCRE2_SIZE startoffset,
                  uint32_t options, pcre2_match_data_8* match_data, pcre2_match_context_8* mcontext);
PCRE2_SIZE* pcre2_get_ovector_pointer_8(pcre2_match_data_8* match_data);
int pcre2_get_error_message_8(int errorcode, PCRE2_UCHAR8* buffer, PCRE2_SIZE bufflen);

#ifdef __cplusplus
}
#endif

#if PCRE2_CODE_UNIT_WIDTH == 8
#define PCRE2_UCHAR PCRE2_UCHAR8
#define PCRE2_SPTR PCRE2_SPTR8
#define pcre2_code pcre2_code_8
#define pcre2_match_data pcre2_match_data_8
#define pcre2_compile pcre2_compile_8
#define pcre2_code_free pcre2_code_free_8
#define pcre2_match_data_create_from_pattern pcre2_match_data_create_from_pattern_8
#define pcre2_match_data_free pcre2_match_data_free_8
#define pcre2_match pcre2_match_8
#define pcre2_get_ovector_pointer pcre2_get_ovector_pointer_8
#define pcre2_get_error_message pcre2_get_error_message_8
#endif

#endif
