#include "kern_table.cuh"
// Kahan summation is a float32-only option (as in the reference), so the double table
// instantiates only the plain segmented reduction.
namespace oeqb { OEQB_DEFINE_DET_TABLE(double, false) }
