#include "kern_table.cuh"
namespace oeqb { OEQB_DEFINE_BATCH_TABLE(float) OEQB_DEFINE_ROW_TABLE(float) OEQB_DEFINE_CW_TABLE(float) }
