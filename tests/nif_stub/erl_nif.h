/* Test infrastructure: the declarations of the Erlang NIF API (erl_nif.h of Erlang/OTP) that
 * c_src/tq4_nif.c uses, with the signatures OTP documents, so that gcc can type-check the NIF
 * against include/tq4.h on a host without Erlang. Nothing is linked or run against it. */
#ifndef TQ4_TEST_ERL_NIF_STUB_H
#define TQ4_TEST_ERL_NIF_STUB_H

#include <stddef.h>
#include <stdint.h>

typedef uint64_t ERL_NIF_TERM;
typedef struct enif_environment_t ErlNifEnv;
typedef struct enif_resource_type_t ErlNifResourceType;
typedef struct ErlDrvMutex ErlNifMutex;
typedef int64_t ErlNifSInt64;
typedef uint64_t ErlNifUInt64;
typedef void ErlNifResourceDtor(ErlNifEnv*, void*);

typedef struct {
  size_t size;
  unsigned char* data;
  void* ref_bin;
  void* __spare__[2];
} ErlNifBinary;

typedef enum { ERL_NIF_LATIN1 = 1 } ErlNifCharEncoding;
typedef enum { ERL_NIF_RT_CREATE = 1, ERL_NIF_RT_TAKEOVER = 2 } ErlNifResourceFlags;
enum { ERL_NIF_DIRTY_JOB_CPU_BOUND = 1, ERL_NIF_DIRTY_JOB_IO_BOUND = 2 };

typedef struct {
  const char* name;
  unsigned arity;
  ERL_NIF_TERM (*fptr)(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]);
  unsigned flags;
} ErlNifFunc;

ErlNifResourceType* enif_open_resource_type(ErlNifEnv*, const char*, const char*, ErlNifResourceDtor*,
                                            ErlNifResourceFlags, ErlNifResourceFlags*);
void* enif_alloc_resource(ErlNifResourceType*, size_t);
void enif_release_resource(void*);
ERL_NIF_TERM enif_make_resource(ErlNifEnv*, void*);
int enif_get_resource(ErlNifEnv*, ERL_NIF_TERM, ErlNifResourceType*, void**);
int enif_get_int(ErlNifEnv*, ERL_NIF_TERM, int*);
int enif_get_int64(ErlNifEnv*, ERL_NIF_TERM, ErlNifSInt64*);
int enif_get_uint64(ErlNifEnv*, ERL_NIF_TERM, ErlNifUInt64*);
int enif_inspect_binary(ErlNifEnv*, ERL_NIF_TERM, ErlNifBinary*);
int enif_get_tuple(ErlNifEnv*, ERL_NIF_TERM, int*, const ERL_NIF_TERM**);
int enif_get_string(ErlNifEnv*, ERL_NIF_TERM, char*, unsigned, ErlNifCharEncoding);
int enif_get_list_length(ErlNifEnv*, ERL_NIF_TERM, unsigned*);
int enif_get_list_cell(ErlNifEnv*, ERL_NIF_TERM, ERL_NIF_TERM*, ERL_NIF_TERM*);
ERL_NIF_TERM enif_make_atom(ErlNifEnv*, const char*);
ERL_NIF_TERM enif_make_int(ErlNifEnv*, int);
ERL_NIF_TERM enif_make_string(ErlNifEnv*, const char*, ErlNifCharEncoding);
ERL_NIF_TERM enif_make_tuple2(ErlNifEnv*, ERL_NIF_TERM, ERL_NIF_TERM);
ERL_NIF_TERM enif_make_badarg(ErlNifEnv*);
ErlNifMutex* enif_mutex_create(char*);
void enif_mutex_destroy(ErlNifMutex*);
void enif_mutex_lock(ErlNifMutex*);
void enif_mutex_unlock(ErlNifMutex*);

typedef struct {
  const char* name;
  ErlNifFunc* funcs;
  int num_of_funcs;
  int (*load)(ErlNifEnv*, void**, ERL_NIF_TERM);
  int (*reload)(ErlNifEnv*, void**, ERL_NIF_TERM);
  int (*upgrade)(ErlNifEnv*, void**, void**, ERL_NIF_TERM);
  void (*unload)(ErlNifEnv*, void*);
} ErlNifEntry;

#define ERL_NIF_INIT(NAME, FUNCS, LOAD, RELOAD, UPGRADE, UNLOAD)                                   \
  const ErlNifEntry* nif_init(void);                                                               \
  const ErlNifEntry* nif_init(void) {                                                              \
    static ErlNifEntry entry = {#NAME, FUNCS, (int)(sizeof(FUNCS) / sizeof(FUNCS[0])), LOAD, RELOAD, \
                                UPGRADE, UNLOAD};                                                  \
    return &entry;                                                                                 \
  }

#endif
