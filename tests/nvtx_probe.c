/* Test-only NVTX injection library: writes every range push and pop of NVTX's default domain in
 * the process as a line "push <name>" or "pop" to the file named by NVTX_PROBE_LOG. NVTX loads it
 * on its first call in a process whose NVTX_INJECTION64_PATH names it, once for each copy of the
 * header-only NVTX in the process (libbolt3.so's, torch's), and calls InitializeInjectionNvtx2,
 * which puts the recording functions into that copy's table of core functions.
 *
 * Build: gcc -shared -fPIC -I<cuda>/include nvtx_probe.c -o nvtx_probe.so (tests/test_trace.py).
 */
#include <stdio.h>
#include <stdlib.h>

#include <nvtx3/nvToolsExt.h>

static FILE* probe_log;

static void probe_line(const char* what, const char* name) {
  if (!probe_log) return;
  if (name) fprintf(probe_log, "%s %s\n", what, name);
  else fprintf(probe_log, "%s\n", what);
  fflush(probe_log);
}

static int probe_push_a(const char* message) {
  probe_line("push", message ? message : "");
  return 0;
}

static int probe_push_ex(const nvtxEventAttributes_t* e) {
  const int ascii = e && e->messageType == NVTX_MESSAGE_TYPE_ASCII && e->message.ascii;
  probe_line("push", ascii ? e->message.ascii : "");
  return 0;
}

static int probe_pop(void) {
  probe_line("pop", NULL);
  return 0;
}

int InitializeInjectionNvtx2(NvtxGetExportTableFunc_t get_export_table) {
  const NvtxExportTableCallbacks* cb = (const NvtxExportTableCallbacks*)get_export_table(NVTX_ETID_CALLBACKS);
  NvtxFunctionTable table = 0;
  unsigned int last = 0; /* the highest valid index of the table */
  if (!cb || !cb->GetModuleFunctionTable) return 0;
  if (!cb->GetModuleFunctionTable(NVTX_CB_MODULE_CORE, &table, &last) || !table) return 0;
  if (last < NVTX_CBID_CORE_RangePop) return 0;
  if (!probe_log) {
    const char* path = getenv("NVTX_PROBE_LOG");
    probe_log = path ? fopen(path, "a") : NULL;
  }
  *table[NVTX_CBID_CORE_RangePushA] = (NvtxFunctionPointer)probe_push_a;
  *table[NVTX_CBID_CORE_RangePushEx] = (NvtxFunctionPointer)probe_push_ex;
  *table[NVTX_CBID_CORE_RangePop] = (NvtxFunctionPointer)probe_pop;
  return 1;
}
