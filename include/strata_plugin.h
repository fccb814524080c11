/*
 * strata_plugin.h — the Ferrite Strata plugin C ABI, version 0.1.
 *
 * A C restatement of the `#[repr(C)]` layouts in the reference's
 * crates/ferrite-strata-plugin-api/src/raw.rs (lines 28-789).  The reference
 * names this header (raw.rs:4, plugin-api/src/lib.rs:17-24) but does not ship
 * it, so every struct below is written field by field, in the same order, from
 * raw.rs.  Rust `Option<unsafe extern "C" fn>` is a nullable C function
 * pointer; `#[repr(u32)]` enums are plain `uint32_t` here so that the width
 * never depends on a C compiler's enum rules.
 *
 * The B200 backend (libstrata_b200.so) exports exactly one symbol,
 * `strata_plugin_v1`, of type `StrataPluginV1` (raw.rs:558-562).
 */
#ifndef STRATA_PLUGIN_H
#define STRATA_PLUGIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- versioning (raw.rs:37-49) ------------------------------------------ */
typedef struct StrataAbiVersion {
  uint32_t major; /* incompatible change: must match exactly            */
  uint32_t minor; /* additive change: host accepts a plugin with higher */
} StrataAbiVersion;

#define STRATA_ABI_MAJOR 0u
#define STRATA_ABI_MINOR 1u

/* ---- extension chain (raw.rs:51-122) ------------------------------------ */
typedef uint32_t StrataExtType;

typedef struct StrataExtBase {
  size_t struct_size; /* size of the whole extension, header included */
  StrataExtType ty;   /* unrecognised values are skipped              */
  struct StrataExtBase *next;
} StrataExtBase;

#define STRATA_EXT_NONE 0u
#define STRATA_EXT_PLUGIN_VERSION 1u /* raw.rs:85  */
#define STRATA_EXT_MESSAGE 2u        /* raw.rs:112 */

typedef struct StrataPluginVersionExt { /* raw.rs:91-104 */
  StrataExtBase base;
  uint16_t major;
  uint16_t minor;
  uint16_t patch;
  StrataAbiVersion targets;
} StrataPluginVersionExt;

typedef struct StrataMessageExt { /* raw.rs:115-122 */
  StrataExtBase base;
  const char *message; /* NUL-terminated UTF-8, owned by the error */
} StrataMessageExt;

/* Opaque handles (raw.rs:132-136, 521-556). */
typedef struct StrataError StrataError;
typedef struct StrataBuffer StrataBuffer;
typedef struct StrataEvent StrataEvent;
typedef struct StrataExecutable StrataExecutable;

/* Returns non-zero to stop iteration (raw.rs:138-146). */
typedef int32_t (*StrataPayloadVisitor)(void *ctx, StrataExtBase *payload);

/* ---- element types (raw.rs:154-185); the hole at 1 is deliberate -------- */
typedef uint32_t StrataElementType;
#define STRATA_ELEM_F8E5M2 0u
#define STRATA_ELEM_F8E4M3 2u
#define STRATA_ELEM_F16 3u
#define STRATA_ELEM_F32 4u
#define STRATA_ELEM_F64 5u
#define STRATA_ELEM_I8 6u
#define STRATA_ELEM_I16 7u
#define STRATA_ELEM_I32 8u
#define STRATA_ELEM_I64 9u
#define STRATA_ELEM_U8 10u
#define STRATA_ELEM_BOOL 11u
#define STRATA_ELEM_F8E8M0 12u
#define STRATA_ELEM_F4E2M1 13u
#define STRATA_ELEM_BF16 14u

/* ---- quantisation (raw.rs:188-227) -------------------------------------- */
typedef uint32_t StrataQuantKind;
#define STRATA_QUANT_NONE 0u
#define STRATA_QUANT_BLOCK 1u
#define STRATA_QUANT_MICROSCALING 2u

typedef struct StrataQuantSpec {
  StrataQuantKind kind;
  uint32_t block_size;
  uint8_t symmetric;
} StrataQuantSpec;

typedef struct StrataDType {
  StrataElementType element;
  StrataQuantSpec quant;
} StrataDType;

/* ---- shape classes (raw.rs:235-272) ------------------------------------- */
typedef uint32_t StrataShapeClassKind;
#define STRATA_SHAPE_SCALAR 0u
#define STRATA_SHAPE_EMPTY 1u
#define STRATA_SHAPE_OUTER_PRODUCT 2u
#define STRATA_SHAPE_VECTOR 3u
#define STRATA_SHAPE_MATRIX 4u
#define STRATA_SHAPE_BATCH3 5u
#define STRATA_SHAPE_BATCH4 6u
#define STRATA_SHAPE_HIGHER_RANK 7u

typedef struct StrataShapeClass {
  StrataShapeClassKind kind;
  uint8_t rank;        /* HigherRank only, zero otherwise */
  uint8_t reserved[2]; /* must be zero                    */
} StrataShapeClass;

/* ---- support levels (raw.rs:275-284) ------------------------------------ */
typedef uint32_t StrataSupportLevel;
#define STRATA_SUPPORT_REFUSE 0u
#define STRATA_SUPPORT_FALLBACK 1u
#define STRATA_SUPPORT_FUSED 2u

/* ---- op tags (raw.rs:294-331) ------------------------------------------- */
typedef uint32_t StrataOpKind;
#define STRATA_OP_INPUT 0u
#define STRATA_OP_ADD 1u
#define STRATA_OP_MUL 2u
#define STRATA_OP_MATMUL 3u
#define STRATA_OP_LOG 4u
#define STRATA_OP_EXP 5u
#define STRATA_OP_SOFTMAX 6u
#define STRATA_OP_LAYER_NORM 7u
#define STRATA_OP_GELU 8u
#define STRATA_OP_LINEAR 9u
#define STRATA_OP_RESHAPE 10u
#define STRATA_OP_TRANSPOSE 11u
#define STRATA_OP_EXPAND 12u
#define STRATA_OP_SLICE 13u
#define STRATA_OP_CUSTOM 14u

/* ---- status codes (status.rs:34-59) ------------------------------------- */
#define STRATA_OK 0
#define STRATA_DECLINED 1
#define STRATA_UNIMPLEMENTED (-2)
#define STRATA_INVALID_ARGUMENT (-3)
#define STRATA_NOT_FOUND (-4)
#define STRATA_RESOURCE_EXHAUSTED (-5)
#define STRATA_INTERNAL (-6) /* the only code that poisons the device */

/* ---- blobs and queries (raw.rs:369-456) --------------------------------- */
typedef struct StrataBlob {
  size_t len;
  const uint8_t *data;
  uint8_t nul;
} StrataBlob;

typedef struct StrataPatternQuery {
  size_t struct_size;
  const uint8_t *pattern_id;
  size_t pattern_id_len;
  StrataDType dtype;
  StrataShapeClass shape_class;
} StrataPatternQuery;

/* b"STRATAG1" as a little-endian u64 (raw.rs:570). */
#define STRATA_WIRE_MAGIC 0x3147415441525453ull
#define STRATA_WIRE_HEADER_LEN 24u
#define STRATA_WIRE_FORMAT_MAJOR 0u
#define STRATA_WIRE_FORMAT_MINOR 1u

typedef struct StrataWireBlob {
  uint64_t magic;
  uint32_t format_major;
  uint32_t format_minor;
  uint64_t payload_len;  /* bytes following the header */
  const uint8_t *data;   /* payload, owned by the producer */
  uint8_t nul;           /* always zero, never counted */
} StrataWireBlob;

typedef struct StrataCompileArgs {
  size_t struct_size;
  StrataWireBlob subgraph;
  const uint8_t *pattern_id; /* advisory; may be null */
  size_t pattern_id_len;
  StrataWireBlob capabilities;
  uint8_t probe; /* do everything except dispatch */
  uint8_t reserved[7];
} StrataCompileArgs;

/* ---- run arguments (raw.rs:458-519) ------------------------------------- */
typedef struct StrataBufferRef {
  StrataBuffer *buffer; /* null means "no buffer" */
  uint32_t value_index; /* index into the decoded subgraph's values */
  uint32_t reserved;
} StrataBufferRef;

typedef struct StrataArenaEntryView {
  uint64_t element_count;
  StrataDType dtype;
  uint8_t *data;
} StrataArenaEntryView;

typedef struct StrataArenaView {
  uint32_t entry_count;
  StrataArenaEntryView *entries;
} StrataArenaView;

typedef struct StrataRunArgs {
  size_t struct_size;
  const StrataExecutable *executable;
  uint32_t arg_count;
  const StrataBufferRef *args;
  StrataArenaView *host_arena; /* null in the normal case */
} StrataRunArgs;

typedef struct StrataAllocDesc {
  size_t struct_size;
  StrataDType dtype;
  uint32_t rank;
  uint32_t reserved;
  const uint64_t *dims;
} StrataAllocDesc;

#define STRATA_PLUGIN_ENTRY_SYMBOL "strata_plugin_v1"

/* ---- the vtable (raw.rs:591-789) ---------------------------------------- */
typedef struct StrataPluginV1 {
  size_t struct_size;
  StrataExtBase *extension_start;
  StrataAbiVersion abi_version;

  /* error handling, mandatory */
  void (*error_free)(StrataError *error);
  uint32_t (*error_code)(const StrataError *error);
  void (*error_payload)(const StrataError *error, StrataPayloadVisitor visitor,
                        void *ctx);

  /* capability, mandatory */
  int32_t (*capabilities)(void *ctx, StrataWireBlob *out);
  uint32_t (*supports)(void *ctx, const StrataPatternQuery *query);

  /* compilation, mandatory */
  int32_t (*compile)(void *ctx, const StrataCompileArgs *args,
                     StrataExecutable **out_executable,
                     StrataError **out_error);

  /* buffers and events */
  int32_t (*alloc)(void *ctx, const StrataAllocDesc *desc,
                   StrataBuffer **out_buffer, StrataError **out_error);
  int32_t (*buffer_release)(void *ctx, StrataBuffer *buffer);
  int32_t (*buffer_write)(void *ctx, StrataBuffer *buffer, uint64_t offset,
                          const uint8_t *data, uint64_t len);
  int32_t (*buffer_read)(void *ctx, const StrataBuffer *buffer,
                         uint64_t offset, uint8_t *data, uint64_t len);
  int32_t (*buffer_event)(void *ctx, const StrataBuffer *buffer,
                          StrataEvent **out_event);
  int32_t (*event_ready)(void *ctx, const StrataEvent *event);
  int32_t (*event_await)(void *ctx, const StrataEvent *event);
  int32_t (*event_free)(void *ctx, StrataEvent *event);

  /* execution, mandatory */
  int32_t (*run)(void *ctx, const StrataRunArgs *args,
                 StrataError **out_error);

  /* teardown, mandatory */
  void (*free_executable)(void *ctx, StrataExecutable *executable);
  void (*free_blob)(void *ctx, StrataWireBlob *blob);
  void *(*plugin_init)(void);
  void (*plugin_free)(void *ctx);

  /* ahead-of-time artefacts, optional */
  int32_t (*serialize)(void *ctx, const StrataExecutable *executable,
                       StrataWireBlob *out_blob);
  int32_t (*deserialize_load)(void *ctx, const StrataWireBlob *blob,
                              StrataExecutable **out_executable);
  int32_t (*abi_compatible)(void *ctx, const StrataWireBlob *blob);
} StrataPluginV1;

#ifdef __cplusplus
} /* extern "C" */
#endif

#if defined(__cplusplus) && defined(__x86_64__)
/* Layout pins for x86-64 (LP64), the platform the Rust host builds for. */
static_assert(sizeof(StrataExtBase) == 24, "StrataExtBase layout");
static_assert(sizeof(StrataPluginVersionExt) == 40, "version ext layout");
static_assert(sizeof(StrataMessageExt) == 32, "message ext layout");
static_assert(sizeof(StrataQuantSpec) == 12, "quant spec layout");
static_assert(sizeof(StrataDType) == 16, "dtype layout");
static_assert(sizeof(StrataShapeClass) == 8, "shape class layout");
static_assert(sizeof(StrataPatternQuery) == 48, "pattern query layout");
static_assert(sizeof(StrataWireBlob) == 40, "wire blob layout");
static_assert(sizeof(StrataCompileArgs) == 112, "compile args layout");
static_assert(sizeof(StrataBufferRef) == 16, "buffer ref layout");
static_assert(sizeof(StrataRunArgs) == 40, "run args layout");
static_assert(sizeof(StrataAllocDesc) == 40, "alloc desc layout");
static_assert(sizeof(StrataPluginV1) == 24 + 22 * 8, "vtable layout");
#endif

#endif /* STRATA_PLUGIN_H */
