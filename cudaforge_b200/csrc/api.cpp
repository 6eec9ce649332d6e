// Status strings and version of the cudaforge_b200 C ABI.
#include "cf_api.h"

extern "C" const char *cf_status_string(int status) {
  switch (status) {
    case CF_OK: return "CF_OK";
    case CF_EINVAL: return "CF_EINVAL: invalid argument";
    case CF_ERANGE: return "CF_ERANGE: index out of range";
    case CF_ETIMEOUT: return "CF_ETIMEOUT: bounded device wait expired";
    case CF_ECUDA: return "CF_ECUDA: CUDA runtime error";
    case CF_ENOMEM: return "CF_ENOMEM: out of memory / KV pages";
    case CF_EUNSUPPORTED: return "CF_EUNSUPPORTED: configuration not supported";
    default: return "unknown cf_status";
  }
}

extern "C" const char *cf_version(void) { return "cudaforge_b200 0.1 sm_100a"; }
