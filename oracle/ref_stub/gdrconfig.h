/* TEST INFRASTRUCTURE ONLY: empty stand-in for GDRCopy's configuration header
 * (see gdrapi.h in this folder). */
#ifndef GOFANN_REF_STUB_GDRCONFIG_H
#define GOFANN_REF_STUB_GDRCONFIG_H
#endif
