#include "kern_table.cuh"
namespace oeqb { OEQB_DEFINE_DET_TABLE(float, true) }
