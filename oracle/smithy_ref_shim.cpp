// C entry points around the reference's header-only smithy loader
// (patches/smithy-config.h, included in place from the reference tree by oracle/Makefile).
// Test infrastructure only: tests load oracle/_ref/libsmithy_ref.so and compare its table
// with libanvil's anvil_smithy_* on the same files.
#include "smithy-config.h"

extern "C" {
int ref_smithy_bucket(int dim) { return (int)smithy_get_bucket(dim); }
void ref_smithy_set_model(const char *path) { smithy_set_model(path); }
int ref_smithy_load(const char *path) {
    std::unique_lock<std::shared_mutex> guard(smithy_load_mutex);
    return smithy_load_configs(path) ? 1 : 0;
}
void ref_smithy_lookup(int type, int nrows, int ncols, int *nw, int *rpb) {
    smithy_shape_config c = smithy_lookup(type, nrows, ncols);
    *nw = c.nwarps;
    *rpb = c.rows_per_block;
}
// Reads one raw table cell regardless of the loaded flag.
void ref_smithy_cell(int type, int nb, int kb, int *nw, int *rpb) {
    *nw = smithy_configs[type][nb][kb].nwarps;
    *rpb = smithy_configs[type][nb][kb].rows_per_block;
}
int ref_smithy_loaded(void) { return smithy_configs_loaded.load() ? 1 : 0; }
void ref_smithy_clear(void) {
    std::unique_lock<std::shared_mutex> guard(smithy_load_mutex);
    memset(smithy_configs, 0, sizeof(smithy_configs));
    smithy_configs_loaded.store(false);
    smithy_load_attempted.store(true);  // no lazy environment load behind the test's back
}
}
