/*
 * Stand-in for <libxsmm.h> so that the reference's scalar contraction path can
 * be compiled from its own sources (TEST INFRASTRUCTURE ONLY, see ref.mk).
 *
 * libxsmm is a third-party dependency that is absent here (the reference's CI
 * clones libxsmm/libxsmm at `main`, pinned to no version). The reference's
 * scalar path reaches this header only through the #include in
 * src/basic/unary/UnaryBackendTpp.h:4, whose class names three libxsmm types
 * as members and return types. This file declares just those three names, as
 * opaque stand-ins; it declares no libxsmm function, and the scalar path calls
 * none (the packing unaries that would use them are never compiled by the
 * scalar backend; ref_scalar.cpp makes any such use fail loudly).
 */
#ifndef EIR_ORACLE_STUB_LIBXSMM_H
#define EIR_ORACLE_STUB_LIBXSMM_H

typedef void (*libxsmm_meltwfunction_unary)(void const *);
typedef void (*libxsmm_meltwfunction_binary)(void const *);
typedef int libxsmm_datatype;

#endif
