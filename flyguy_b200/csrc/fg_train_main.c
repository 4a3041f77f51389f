/* The fg_train executable: the standalone teaching trainer of libflyguy_b200.so (fg_train_main; usage there). */
#include "flyguy_b200.h"

int main(int argc, char** argv) { return fg_train_main(argc, (const char* const*)argv); }
