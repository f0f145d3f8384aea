// powerbench: the command-line front end of libpmb200's workload engine.
// Same flags and JSONL stdout as the reference's powerbench; errors go to
// stderr as "powerbench: <msg>" with exit status 1.
#include <cstdio>
#include <cstring>

#include "pmb200.h"

static void print_line(const char* line, void*) {
  if (line[0] == '#') { fputs(line + 1, stdout); fflush(stdout); return; }   // --help text
  fputs(line, stdout);
  fputc('\n', stdout);
  fflush(stdout);
}

int main(int argc, char** argv) {
  const int rc = pm_powerbench(argc, const_cast<const char* const*>(argv), print_line, nullptr);
  if (rc != 0) {
    char msg[2048];
    pm_last_error(msg, sizeof msg);
    fprintf(stderr, "powerbench: %s\n", msg);
    return 1;
  }
  return 0;
}
